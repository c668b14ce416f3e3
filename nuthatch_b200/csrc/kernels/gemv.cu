// Batch-1 GEMV kernels over native GGUF Q4_K / Q6_K / F32 rows.
//
// Layout of the work: the activation row is prepared once per CTA in shared
// memory (optional RMSNorm, Q8_K quantisation).  Each warp owns a sequence of
// jobs; a job is a group of consecutive weight rows (32/lanes_per_row rows)
// staged into the warp's shared buffer with 16-byte cp.async copies,
// kernels_stages deep, so several KB per warp are in flight while the previous
// group is reduced.  Within a group one lane handles one super-block of one
// row; the lanes of a row reduce with shuffles.
#include <climits>

#include "common.cuh"

namespace nh {

constexpr int kGemvWarps = 4;
constexpr int kGemvStages = 3;
constexpr int kMaxArgmaxBlocks = 2048;

struct GemvSeg {
  const uint8_t* w;
  float* out;
  const float* resid;
  int32_t rows;
  int32_t type;
  uint64_t rb;
};

struct GemvArgs {
  GemvSeg seg[3];
  int nseg;
  int K;
  int lpr;  // lanes per row for quantised segments
  int rpp;  // rows per job for quantised segments (32 / lpr)
  int jobs_start[4];
  int jobs_total;
  uint32_t stage_bytes;
  const float* x;
  const float* norm_w;
  float eps;
  int do_norm;
  int quant;
  // lm_head argmax mode
  int argmax;
  NhDecodeState* state;
  float* part_val;
  int32_t* part_idx;
  unsigned* ticket;
  int32_t* out_tokens;
  float* logits_dump;
};

__device__ __forceinline__ void gemv_job(const GemvArgs& p, int j, int& s, int& row0, int& nrows) {
  s = 0;
  while (s + 1 < p.nseg && j >= p.jobs_start[s + 1]) ++s;
  const int rpp = p.seg[s].type == NH_TYPE_F32 ? 1 : p.rpp;
  row0 = (j - p.jobs_start[s]) * rpp;
  nrows = min(rpp, p.seg[s].rows - row0);
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.K);
  const size_t act_bytes = (act_smem_bytes(p.K) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  uint8_t* stage = smem + act_bytes + 48 * sizeof(double);
  __shared__ float s_bv[kGemvWarps];
  __shared__ int s_bi[kGemvWarps];
  __shared__ bool s_last;

  int pos = 0, n_prompt = 0;
  bool skip = false;
  if (p.argmax) {
    pos = p.state->pos;
    n_prompt = p.state->n_prompt;
    skip = pos < n_prompt - 1;
  }
  float best_v = -INFINITY;
  int best_i = INT_MAX;
  if (!skip) {
    prep_act(a, p.x, p.norm_w, p.do_norm != 0, p.eps, p.quant != 0, red);
    const int gw = blockIdx.x * kGemvWarps + warp;
    const int tw = gridDim.x * kGemvWarps;
    uint8_t* wb = stage + static_cast<size_t>(warp) * kGemvStages * p.stage_bytes;
    const int nsb = p.K / QK;
    const int sub = lane % p.lpr, kr = lane / p.lpr;

    auto issue = [&](int j, uint8_t* buf) {
      int s, row0, nrows;
      gemv_job(p, j, s, row0, nrows);
      if (p.seg[s].type == NH_TYPE_F32) return;
      stage_bytes_warp(buf, p.seg[s].w + static_cast<uint64_t>(row0) * p.seg[s].rb,
                       static_cast<size_t>(nrows) * p.seg[s].rb, lane);
    };
#pragma unroll
    for (int st = 0; st < kGemvStages; ++st) {
      const int j = gw + st * tw;
      if (j < p.jobs_total) issue(j, wb + st * p.stage_bytes);
      cp_async_commit();
    }
    for (int it = 0;; ++it) {
      const int j = gw + it * tw;
      if (j >= p.jobs_total) break;
      cp_async_wait<kGemvStages - 1>();
      __syncwarp();
      uint8_t* buf = wb + (it % kGemvStages) * p.stage_bytes;
      int s, row0, nrows;
      gemv_job(p, j, s, row0, nrows);
      const GemvSeg& sg = p.seg[s];
      float v;
      int r;
      bool writer;
      if (sg.type == NH_TYPE_F32) {
        r = row0;
        v = row_dot_f32(reinterpret_cast<const float*>(sg.w + static_cast<uint64_t>(r) * sg.rb),
                        a.xf, p.K, lane);
        writer = lane == 0;
      } else {
        const uintptr_t off = reinterpret_cast<uintptr_t>(sg.w + static_cast<uint64_t>(row0) * sg.rb) & 15;
        const uint8_t* rowp = buf + off + static_cast<size_t>(kr) * sg.rb;
        v = row_dot_q(rowp, sg.type, nsb, sub, p.lpr, a);
        r = row0 + kr;
        writer = sub == 0 && kr < nrows;
      }
      if (writer) {
        if (sg.resid != nullptr) v = __fadd_rn(sg.resid[r], v);
        if (sg.out != nullptr) sg.out[r] = v;
        if (p.argmax) {
          if (p.logits_dump != nullptr) {
            p.logits_dump[static_cast<int64_t>(pos - n_prompt + 1) * sg.rows + r] = v;
          }
          if (better(v, r, best_v, best_i)) {
            best_v = v;
            best_i = r;
          }
        }
      }
      __syncwarp();
      const int jn = gw + (it + kGemvStages) * tw;
      if (jn < p.jobs_total) issue(jn, buf);
      cp_async_commit();
    }
    cp_async_wait<0>();
  }
  if (!p.argmax) return;

  // Block argmax, then the last CTA (by ticket) reduces the per-CTA partials
  // and advances the decode cursor.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (better(ov, oi, best_v, best_i)) {
      best_v = ov;
      best_i = oi;
    }
  }
  if (lane == 0) {
    s_bv[warp] = best_v;
    s_bi[warp] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bv = s_bv[0];
    int bi = s_bi[0];
    for (int w = 1; w < kGemvWarps; ++w)
      if (better(s_bv[w], s_bi[w], bv, bi)) {
        bv = s_bv[w];
        bi = s_bi[w];
      }
    p.part_val[blockIdx.x] = bv;
    p.part_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned t = atomicAdd(p.ticket, 1u);
    s_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  if (!skip) {
    volatile float* pv = p.part_val;
    volatile int32_t* pi = p.part_idx;
    float bv = pv[0];
    int bi = pi[0];
    for (unsigned b = 1; b < gridDim.x; ++b)
      if (better(pv[b], pi[b], bv, bi)) {
        bv = pv[b];
        bi = pi[b];
      }
    if (bi == INT_MAX) bi = 0;
    const int n = p.state->n_out;
    if (n < p.state->n_predict) p.out_tokens[n] = bi;
    p.state->token = bi;
    p.state->n_out = n + 1;
  }
  p.state->pos = pos + 1;
  *p.ticket = 0u;
}

namespace {

int g_sm_count[16] = {0};

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) dev = 0;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

bool valid_type(int t) { return t == NH_TYPE_F32 || t == NH_TYPE_Q4_K || t == NH_TYPE_Q6_K; }

// Fills the work split of a GemvArgs whose segments, K and activation source are set.
int gemv_launch(GemvArgs& p, cudaStream_t stream) {
  if (p.K <= 0 || p.K > kMaxK) return NH_E_ARG;
  bool any_q = false;
  uint64_t rb_max = 0;
  for (int s = 0; s < p.nseg; ++s) {
    if (!valid_type(p.seg[s].type) || p.seg[s].w == nullptr || p.seg[s].rows < 0) return NH_E_ARG;
    if (p.seg[s].type != NH_TYPE_F32) {
      if (p.K % QK != 0) return NH_E_ARG;
      any_q = true;
    }
    p.seg[s].rb = row_bytes(p.seg[s].type, p.K);
    rb_max = rb_max > p.seg[s].rb ? rb_max : p.seg[s].rb;
  }
  p.quant = any_q ? 1 : 0;
  p.lpr = any_q ? lanes_per_row(p.K / QK) : 32;
  p.rpp = 32 / p.lpr;
  int total = 0;
  for (int s = 0; s < p.nseg; ++s) {
    p.jobs_start[s] = total;
    const int rpp = p.seg[s].type == NH_TYPE_F32 ? 1 : p.rpp;
    total += (p.seg[s].rows + rpp - 1) / rpp;
  }
  for (int s = p.nseg; s < 4; ++s) p.jobs_start[s] = total;
  p.jobs_total = total;
  p.stage_bytes = any_q ? static_cast<uint32_t>((rb_max * p.rpp + 32 + 15) & ~15ull) : 16u;
  const size_t smem = ((act_smem_bytes(p.K) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double) +
                      static_cast<size_t>(kGemvWarps) * kGemvStages * p.stage_bytes;
  static size_t configured = 0;
  if (smem > configured) {
    if (cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
      return NH_E_CUDA;
    }
    configured = smem;
  }
  const int per_sm = smem > 110 * 1024 ? 1 : 2;
  int grid = (total + kGemvWarps - 1) / kGemvWarps;
  const int cap = sm_count() * per_sm;
  if (grid > cap) grid = cap;
  if (p.argmax && grid > kMaxArgmaxBlocks) grid = kMaxArgmaxBlocks;
  if (grid < 1) grid = 1;
  gemv_kernel<<<grid, kGemvWarps * 32, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

GemvArgs blank_args() {
  GemvArgs p;
  memset(&p, 0, sizeof(p));
  return p;
}

}  // namespace
}  // namespace nh

using namespace nh;

extern "C" int nh_device_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return NH_E_CUDA;
  return n;
}

extern "C" int64_t nh_argmax_scratch_bytes(int /*n_vocab*/) {
  return static_cast<int64_t>(kMaxArgmaxBlocks) * 8 + 64;
}

extern "C" int nh_qkv_proj(const float* h, const float* attn_norm, float eps, const void* wq,
                           int32_t tq, const void* wk, int32_t tk, const void* wv, int32_t tv,
                           int64_t n_embd, int64_t n_embd_kv, float* q_out, float* k_out,
                           float* v_out, void* stream) {
  if (h == nullptr || q_out == nullptr || k_out == nullptr || v_out == nullptr) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 3;
  p.K = static_cast<int>(n_embd);
  p.seg[0] = {static_cast<const uint8_t*>(wq), q_out, nullptr, static_cast<int32_t>(n_embd), tq, 0};
  p.seg[1] = {static_cast<const uint8_t*>(wk), k_out, nullptr, static_cast<int32_t>(n_embd_kv), tk, 0};
  p.seg[2] = {static_cast<const uint8_t*>(wv), v_out, nullptr, static_cast<int32_t>(n_embd_kv), tv, 0};
  p.x = h;
  p.norm_w = attn_norm;
  p.eps = eps;
  p.do_norm = 1;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nh_out_proj_residual(const float* x, const void* wo, int32_t to, int64_t n_embd,
                                    float* h_io, void* stream) {
  if (x == nullptr || h_io == nullptr) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 1;
  p.K = static_cast<int>(n_embd);
  p.seg[0] = {static_cast<const uint8_t*>(wo), h_io, h_io, static_cast<int32_t>(n_embd), to, 0};
  p.x = x;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nh_lm_head_argmax(NhDecodeState* state, const float* h, const float* out_norm,
                                 float eps, const void* w, int32_t tw, int64_t n_embd,
                                 int64_t n_vocab, int32_t* out_tokens, float* logits_dump,
                                 void* scratch, void* stream) {
  if (state == nullptr || h == nullptr || out_tokens == nullptr || scratch == nullptr) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 1;
  p.K = static_cast<int>(n_embd);
  p.seg[0] = {static_cast<const uint8_t*>(w), nullptr, nullptr, static_cast<int32_t>(n_vocab), tw, 0};
  p.x = h;
  p.norm_w = out_norm;
  p.eps = eps;
  p.do_norm = 1;
  p.argmax = 1;
  p.state = state;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  p.ticket = reinterpret_cast<unsigned*>(sc);
  p.part_val = reinterpret_cast<float*>(sc + 64);
  p.part_idx = reinterpret_cast<int32_t*>(sc + 64 + kMaxArgmaxBlocks * 4);
  p.out_tokens = out_tokens;
  p.logits_dump = logits_dump;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nh_gemv(const void* w, int32_t type, int64_t n, int64_t rows, const float* x,
                       const float* norm_w, float eps, float* y, void* stream) {
  if (w == nullptr || x == nullptr || y == nullptr || rows <= 0) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 1;
  p.K = static_cast<int>(n);
  p.seg[0] = {static_cast<const uint8_t*>(w), y, nullptr, static_cast<int32_t>(rows), type, 0};
  p.x = x;
  p.norm_w = norm_w;
  p.eps = eps;
  p.do_norm = norm_w != nullptr ? 1 : 0;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

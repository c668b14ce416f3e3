// Batch-1 GEMV kernels over native GGUF Q4_K / Q6_K / F32 rows: QKV,
// output projection + residual, lm_head + argmax, and the standalone form.
//
// Each warp owns a sequence of jobs (a job = 32/LPR consecutive rows of one
// weight), staged by its own cp.async.bulk ring (rowdot.cuh).  The weights do
// not depend on the preceding kernel, so the first kStages jobs are issued
// before griddepcontrol.wait: the HBM stream of this kernel overlaps the tail
// of the previous one.  The activation (optional RMSNorm, Q8_K) is prepared
// once per CTA in shared memory and then held in registers.
#include <climits>
#include <cstring>

#include "launch.cuh"
#include "gemv3.cuh"

namespace nh {

template <int CPL>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const GemvArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.K, true, p.need_wf != 0);
  const size_t act_bytes = (act_smem_bytes(p.K, true, p.need_wf != 0) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes + 48 * sizeof(double));
  uint8_t* stage = smem + act_bytes + 48 * sizeof(double) + kGemvWarps * p.S * sizeof(uint64_t);
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  __shared__ bool s_last;

  int pos = 0, n_prompt = 0;
  bool skip = false;
  if (p.argmax) {
    // The cursor was last written by the previous token's argmax, which has
    // completed before this kernel could launch.
    pos = *reinterpret_cast<volatile const int*>(&p.state->pos);
    n_prompt = *reinterpret_cast<volatile const int*>(&p.state->n_prompt);
    skip = pos < n_prompt - 1;
  }
  const int gw = blockIdx.x * kGemvWarps + warp;
  const int tw = gridDim.x * kGemvWarps;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  auto issue = [&](int j, int st) {
    int s, row0, nrows;
    gemv_job(p, j, s, row0, nrows);
    if (p.seg[s].type == NH_TYPE_F32) return;
    if (lane == 0) {
      uint32_t len, off;
      const uint8_t* src = span16(p.seg[s].w + static_cast<uint64_t>(row0) * p.seg[s].rb,
                                  static_cast<size_t>(nrows) * p.seg[s].rb, &len, &off);
      mbar_expect_tx(&wbar[st], len);
      bulk_g2s(wb + static_cast<size_t>(st) * p.stage_bytes, src, len, &wbar[st]);
    }
  };
  if (!skip) {
#pragma unroll
    for (int st = 0; st < p.S; ++st) {
      const int j = gw + st * tw;
      if (j < p.jobs_total) issue(j, st);
    }
    act_load_norm(a, p.norm_w);
  }
  pdl_wait();
  pdl_trigger();

  float best_v = -INFINITY;
  int best_i = INT_MAX;
  bool failed = false;
  if (!skip) {
    prep_act(a, p.x, p.norm_w != nullptr, p.do_norm != 0, p.eps, p.quant != 0, red);
    const int jl = lane % p.lpr, kr = lane / p.lpr;
    ActReg<CPL> ar;
    if (p.quant) load_act<CPL>(ar, a, 0, jl, p.lpr);
    for (int it = 0;; ++it) {
      const int j = gw + it * tw;
      if (j >= p.jobs_total) break;
      const int st = it % p.S;
      int s, row0, nrows;
      gemv_job(p, j, s, row0, nrows);
      const GemvSeg& sg = p.seg[s];
      float v;
      int r;
      bool writer;
      if (sg.type == NH_TYPE_F32) {
        r = row0;
        v = row_dot_f32(reinterpret_cast<const float*>(sg.w + static_cast<uint64_t>(r) * sg.rb), a.xf, p.K, lane);
        writer = lane == 0;
      } else {
        if (!mbar_wait(&wbar[st], (it / p.S) & 1)) {
          failed = true;
          break;
        }
        const uint32_t off =
            static_cast<uint32_t>(reinterpret_cast<uintptr_t>(sg.w + static_cast<uint64_t>(row0) * sg.rb) & 15);
        const uint8_t* rowp = wb + static_cast<size_t>(st) * p.stage_bytes + off + static_cast<size_t>(kr) * sg.rb;
        v = row_dot_reg<CPL>(rowp, sg.type, jl, p.lpr, ar);
        r = row0 + kr;
        writer = jl == 0 && kr < nrows;
      }
      if (writer) {
        if (sg.resid != nullptr) v = __fadd_rn(sg.resid[r], v);
        if (sg.out != nullptr) sg.out[r] = v;
        if (p.argmax) {
          if (p.logits_dump != nullptr) p.logits_dump[static_cast<int64_t>(pos - n_prompt + 1) * sg.rows + r] = v;
          if (argmax_better(v, r, best_v, best_i)) {
            best_v = v;
            best_i = r;
          }
        }
      }
      __syncwarp();
      const int jn = gw + (it + p.S) * tw;
      if (jn < p.jobs_total) issue(jn, st);
    }
  }
  if (failed && lane == 0 && p.state != nullptr) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  if (!p.argmax) return;

  // Per-CTA argmax, then the last CTA (by ticket) reduces the partials with
  // all its threads and advances the decode cursor.
  block_argmax(best_v, best_i, s_bv, s_bi);
  if (threadIdx.x == 0) {
    p.part_val[blockIdx.x] = best_v;
    p.part_idx[blockIdx.x] = best_i;
    __threadfence();
    const unsigned t = atomicAdd(p.ticket, 1u);
    s_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (!skip) {
    const volatile float* pv = p.part_val;
    const volatile int32_t* pi = p.part_idx;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
      const float v = pv[b];
      const int i = pi[b];
      if (argmax_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
  block_argmax(bv, bi, s_bv, s_bi);
  if (threadIdx.x != 0) return;
  if (!skip) {
    if (bi == INT_MAX) bi = 0;
    const int n = p.state->n_out;
    if (n < p.state->n_predict) p.out_tokens[n] = bi;
    p.state->token = bi;
    p.state->n_out = n + 1;
  }
  p.state->pos = pos + 1;
  *p.ticket = 0u;
}

// Lane-per-super-block form (K <= 2048, every segment quantised): a job is
// P = 32/G rows of one segment, all computed in one warp pass.
__global__ void __launch_bounds__(kGemvWarps * 32, 2) gemv3_kernel(const GemvArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const unsigned ph_idx = phase_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.K, true, p.need_wf != 0);
  const size_t act_bytes = (act_smem_bytes(p.K, true, p.need_wf != 0) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes + 48 * sizeof(double));
  uint8_t* stage = smem + act_bytes + 48 * sizeof(double) + kGemvWarps * p.S * sizeof(uint64_t);
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  __shared__ bool s_last;

  int pos = 0, n_prompt = 0;
  bool skip = false;
  if (p.argmax) {
    pos = *reinterpret_cast<volatile const int*>(&p.state->pos);
    n_prompt = *reinterpret_cast<volatile const int*>(&p.state->n_prompt);
    skip = pos < n_prompt - 1;
  }
  const int gw = blockIdx.x * kGemvWarps + warp;
  const int tw = gridDim.x * kGemvWarps;
  const int G = p.lpr, P = p.rpp;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  auto job = [&](int j, int& s, int& row0, int& nrows) {
    s = 0;
    while (s + 1 < p.nseg && j >= p.jobs_start[s + 1]) ++s;
    row0 = (j - p.jobs_start[s]) * P;
    nrows = min(P, p.seg[s].rows - row0);
  };
  auto issue = [&](int j, int st) {
    if (lane != 0) return;
    int s, row0, nrows;
    job(j, s, row0, nrows);
    uint32_t len, off;
    const uint8_t* src = span16(p.seg[s].w + static_cast<uint64_t>(row0) * p.seg[s].rb,
                                static_cast<size_t>(nrows) * p.seg[s].rb, &len, &off);
    mbar_expect_tx(&wbar[st], len);
    bulk_g2s(wb + static_cast<size_t>(st) * p.stage_bytes, src, len, &wbar[st]);
  };
  if (!skip) {
    for (int st = 0; st < p.S; ++st) {
      const int j = gw + st * tw;
      if (j < p.jobs_total) issue(j, st);
    }
    act_load_norm(a, p.norm_w);
  }
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();

  float best_v = -INFINITY;
  int best_i = INT_MAX;
  bool failed = false;
  if (!skip) {
    prep_act(a, p.x, p.norm_w != nullptr, p.do_norm != 0, p.eps, true, red);
    phase_stamp(2);
    const int g = lane % G, r = lane / G;
    // Most warps dot one or two jobs: the activation is read from shared
    // memory rather than held in registers.
    const Act3Smem act{a, g};
    for (int it = 0;; ++it) {
      const int j = gw + it * tw;
      if (j >= p.jobs_total) break;
      const int st = it % p.S;
      int s, row0, nrows;
      job(j, s, row0, nrows);
      const GemvSeg& sg = p.seg[s];
      if (!mbar_wait(&wbar[st], (it / p.S) & 1)) {
        failed = true;
        break;
      }
      if (it == 0) phase_stamp(3);
      const uint32_t off =
          static_cast<uint32_t>(reinterpret_cast<uintptr_t>(sg.w + static_cast<uint64_t>(row0) * sg.rb) & 15);
      const uint8_t* rowp = wb + static_cast<size_t>(st) * p.stage_bytes + off + static_cast<size_t>(r) * sg.rb;
      float v = row_dot3v(rowp, sg.type, g, G, act);
      const int row = row0 + r;
      if (g == 0 && r < nrows) {
        if (sg.resid != nullptr) v = __fadd_rn(sg.resid[row], v);
        if (sg.out != nullptr) sg.out[row] = v;
        if (p.argmax) {
          if (p.logits_dump != nullptr) p.logits_dump[static_cast<int64_t>(pos - n_prompt + 1) * sg.rows + row] = v;
          if (argmax_better(v, row, best_v, best_i)) {
            best_v = v;
            best_i = row;
          }
        }
      }
      __syncwarp();
      const int jn = gw + (it + p.S) * tw;
      if (jn < p.jobs_total) issue(jn, st);
    }
  }
  phase_end_sync(p.argmax ? kPhLmHead : kPhQkvOrOut, ph_idx);
  if (failed && lane == 0 && p.state != nullptr) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  if (!p.argmax) return;

  block_argmax(best_v, best_i, s_bv, s_bi);
  if (threadIdx.x == 0) {
    p.part_val[blockIdx.x] = best_v;
    p.part_idx[blockIdx.x] = best_i;
    __threadfence();
    const unsigned t = atomicAdd(p.ticket, 1u);
    s_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (!skip) {
    const volatile float* pv = p.part_val;
    const volatile int32_t* pi = p.part_idx;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
      const float v = pv[b];
      const int i = pi[b];
      if (argmax_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
  block_argmax(bv, bi, s_bv, s_bi);
  if (threadIdx.x != 0) return;
  if (!skip) {
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

bool valid_type(int t) { return t == NH_TYPE_F32 || t == NH_TYPE_Q4_K || t == NH_TYPE_Q6_K; }

template <int CPL>
int gemv_launch_t(GemvArgs& p, size_t smem, int grid, cudaStream_t stream) {
  static SmemLimit configured;
  if (!ensure_smem(gemv_kernel<CPL>, smem, configured)) return NH_E_CUDA;
  return launch_pdl(gemv_kernel<CPL>, dim3(grid), dim3(kGemvWarps * 32), smem, stream, p);
}

// Fills the work split of a GemvArgs whose segments, K and activation source are set.
// Resident CTAs per SM for a kernel at a dynamic shared-memory size (at most 4).
template <typename Kern>
int resident_ctas(Kern k, int threads, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess || n < 1) n = 1;
  return n > 4 ? 4 : n;
}

// The lane-per-super-block path: every segment quantised and K <= 2048.
int gemv3_launch(GemvArgs& p, cudaStream_t stream) {
  gemv3_shape(p);
  const int total = p.jobs_total;
  const size_t fixed = ((act_smem_bytes(p.K, true, p.need_wf != 0) + 15) & ~static_cast<size_t>(15)) +
                       48 * sizeof(double);
  p.S = kGemvMaxStages;
  while (p.S > 1 && fixed + static_cast<size_t>(kGemvWarps) * p.S * (p.stage_bytes + 8) > 110 * 1024) --p.S;
  const size_t smem = fixed + kGemvWarps * p.S * sizeof(uint64_t) + static_cast<size_t>(kGemvWarps) * p.S * p.stage_bytes;
  static SmemLimit configured;
  if (!ensure_smem(gemv3_kernel, smem, configured)) return NH_E_CUDA;
  const int per_sm = std::min(resident_ctas(gemv3_kernel, kGemvWarps * 32, smem), ctas_per_sm_cap());
  int grid = (total + kGemvWarps - 1) / kGemvWarps;
  const int cap = device_sm_count() * per_sm;
  if (grid > cap) grid = cap;
  if (p.argmax && grid > kMaxArgmaxBlocks) grid = kMaxArgmaxBlocks;
  if (grid < 1) grid = 1;
  return launch_pdl(gemv3_kernel, dim3(grid), dim3(kGemvWarps * 32), smem, stream, p);
}

int gemv_launch(GemvArgs& p, cudaStream_t stream) {
  if (p.K <= 0 || p.K > kMaxK) return NH_E_ARG;
  {
    bool v3 = rowdot3_k_ok(p.K) && engine_v3();
    for (int s = 0; s < p.nseg; ++s) {
      if (!valid_type(p.seg[s].type) || p.seg[s].w == nullptr || p.seg[s].rows < 0) return NH_E_ARG;
      if (p.seg[s].type == NH_TYPE_F32) v3 = false;
      if (p.seg[s].type == NH_TYPE_Q4_K && (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) != 0) return NH_E_ARG;
    }
    if (v3) return gemv3_launch(p, stream);
  }
  bool any_q = false;
  uint64_t rb_max = 0;
  for (int s = 0; s < p.nseg; ++s) {
    if (!valid_type(p.seg[s].type) || p.seg[s].w == nullptr || p.seg[s].rows < 0) return NH_E_ARG;
    if (p.seg[s].type != NH_TYPE_F32) {
      if (!rowdot_k_ok(p.K)) return NH_E_ARG;
      any_q = true;
    }
    p.seg[s].rb = row_bytes(p.seg[s].type, p.K);
    rb_max = rb_max > p.seg[s].rb ? rb_max : p.seg[s].rb;
  }
  p.quant = any_q ? 1 : 0;
  p.need_wf = (p.do_norm != 0 && p.norm_w != nullptr) ? 1 : 0;
  p.lpr = any_q ? rowdot_lpr(p.K) : 32;
  p.rpp = 32 / p.lpr;
  int total = 0;
  for (int s = 0; s < p.nseg; ++s) {
    p.jobs_start[s] = total;
    const int rpp = p.seg[s].type == NH_TYPE_F32 ? 1 : p.rpp;
    total += (p.seg[s].rows + rpp - 1) / rpp;
  }
  for (int s = p.nseg; s < 4; ++s) p.jobs_start[s] = total;
  p.jobs_total = total;
  p.stage_bytes = any_q ? static_cast<uint32_t>((rb_max * p.rpp + 32 + 127) & ~127ull) : 128u;
  p.S = kGemvMaxStages;
  while (p.S > 2 && static_cast<size_t>(kGemvWarps) * p.S * p.stage_bytes > 96 * 1024) --p.S;
  const size_t smem = ((act_smem_bytes(p.K, true, p.need_wf != 0) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double) +
                      kGemvWarps * p.S * sizeof(uint64_t) +
                      static_cast<size_t>(kGemvWarps) * p.S * p.stage_bytes;
  const int per_sm = static_cast<int>(std::min<size_t>(4, (220 * 1024) / (smem + 1024)));
  int grid = (total + kGemvWarps - 1) / kGemvWarps;
  const int cap = device_sm_count() * (per_sm < 1 ? 1 : per_sm);
  if (grid > cap) grid = cap;
  if (p.argmax && grid > kMaxArgmaxBlocks) grid = kMaxArgmaxBlocks;
  if (grid < 1) grid = 1;
  const int cpl = any_q ? (p.K / 64 + 31) / 32 : 1;
  if (cpl <= 1) return gemv_launch_t<1>(p, smem, grid, stream);
  return gemv_launch_t<2>(p, smem, grid, stream);
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

extern "C" int64_t nh_argmax_scratch_bytes(int /*n_vocab*/) { return static_cast<int64_t>(kMaxArgmaxBlocks) * 8 + 64; }

extern "C" int nh_qkv_proj(NhDecodeState* state, const float* h, const float* attn_norm, float eps, const void* wq, int32_t tq,
                           const void* wk, int32_t tk, const void* wv, int32_t tv, int64_t n_embd, int64_t n_embd_kv,
                           float* q_out, float* k_out, float* v_out, void* stream) {
  if (h == nullptr || q_out == nullptr || k_out == nullptr || v_out == nullptr) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 3;
  p.K = static_cast<int>(n_embd);
  p.seg[0] = {static_cast<const uint8_t*>(wq), q_out, nullptr, static_cast<int32_t>(n_embd), tq, 0};
  p.seg[1] = {static_cast<const uint8_t*>(wk), k_out, nullptr, static_cast<int32_t>(n_embd_kv), tk, 0};
  p.seg[2] = {static_cast<const uint8_t*>(wv), v_out, nullptr, static_cast<int32_t>(n_embd_kv), tv, 0};
  p.state = state;
  p.x = h;
  p.norm_w = attn_norm;
  p.eps = eps;
  p.do_norm = 1;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nh_out_proj_residual(NhDecodeState* state, const float* x, const void* wo, int32_t to, int64_t n_embd, float* h_io,
                                    void* stream) {
  if (x == nullptr || h_io == nullptr) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 1;
  p.K = static_cast<int>(n_embd);
  p.seg[0] = {static_cast<const uint8_t*>(wo), h_io, h_io, static_cast<int32_t>(n_embd), to, 0};
  p.state = state;
  p.x = x;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" int nh_lm_head_argmax(NhDecodeState* state, const float* h, const float* out_norm, float eps, const void* w,
                                 int32_t tw, int64_t n_embd, int64_t n_vocab, int32_t* out_tokens, float* logits_dump,
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

extern "C" int nh_gemv(NhDecodeState* state, const void* w, int32_t type, int64_t n, int64_t rows, const float* x, const float* norm_w,
                       float eps, float* y, void* stream) {
  if (w == nullptr || x == nullptr || y == nullptr || rows <= 0) return NH_E_ARG;
  GemvArgs p = blank_args();
  p.nseg = 1;
  p.K = static_cast<int>(n);
  p.seg[0] = {static_cast<const uint8_t*>(w), y, nullptr, static_cast<int32_t>(rows), type, 0};
  p.state = state;
  p.x = x;
  p.norm_w = norm_w;
  p.eps = eps;
  p.do_norm = norm_w != nullptr ? 1 : 0;
  return gemv_launch(p, static_cast<cudaStream_t>(stream));
}

NH_PHASE_TRACE_SETTER(gemv)

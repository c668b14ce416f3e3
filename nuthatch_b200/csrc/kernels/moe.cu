// MoE kernels for one decode position: router top-k, expert gate/up with
// SwiGLU, expert down projection with the weighted top-k-order combine.
//
// Expert weights are addressed as base + wsel[i] * nb2 (+ row * row_bytes),
// so the same kernels read the resident fused expert tensors or the HBM slot
// pool of the streaming path (where wsel holds slot indices).
#include <climits>

#include "common.cuh"

namespace nh {

constexpr int kMoeWarps = 4;
constexpr int kMoeStages = 3;
constexpr int kRouterWarps = 8;
constexpr int kMaxTopK = 32;

int moe_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ------------------------------------------------------------------ router
struct RouterArgs {
  const NhDecodeState* state;
  const float* h;
  const float* norm;
  float eps;
  const float* router;
  int K, E, topk, norm_topk, layer, n_layers;
  int32_t* sel;
  float* wts;
  int32_t* trace_sel;
  float* trace_gap;
  unsigned* ticket;
  float* logits;
};

__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(const RouterArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  ActSmem a = carve_act(smem, p.K);
  __shared__ double red[48];
  __shared__ bool s_last;
  prep_act(a, p.h, p.norm, true, p.eps, false, red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouterWarps + warp;
  if (e < p.E) {
    const float v = row_dot_f32(p.router + static_cast<int64_t>(e) * p.K, a.xf, p.K, lane);
    if (lane == 0) p.logits[e] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  // ggml_soft_max: exp(x - max) summed in double, scaled by 1/sum.
  volatile float* lg = p.logits;
  float pr[256];
  const int E = p.E;
  float mx = -INFINITY;
  for (int i = 0; i < E; ++i) mx = fmaxf(mx, lg[i]);
  double sum = 0.0;
  for (int i = 0; i < E; ++i) {
    pr[i] = expf(__fsub_rn(lg[i], mx));
    sum += static_cast<double>(pr[i]);
  }
  const float inv = static_cast<float>(1.0 / sum);
  for (int i = 0; i < E; ++i) pr[i] = __fmul_rn(pr[i], inv);
  // Top-k in descending probability; equal probabilities keep the lower id first.
  uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int ids[kMaxTopK + 1];
  const int kk = min(p.topk + 1, E);
  for (int t = 0; t < kk; ++t) {
    int b = -1;
    for (int i = 0; i < E; ++i) {
      if (taken[i >> 5] & (1u << (i & 31))) continue;
      if (b < 0 || pr[i] > pr[b]) b = i;
    }
    ids[t] = b;
    taken[b >> 5] |= 1u << (b & 31);
  }
  float w[kMaxTopK];
  for (int t = 0; t < p.topk; ++t) w[t] = pr[ids[t]];
  if (p.norm_topk) {
    double s = 0.0;
    for (int t = 0; t < p.topk; ++t) s += static_cast<double>(w[t]);
    const float ws = fmaxf(static_cast<float>(s), 6.103515625e-5f);
    for (int t = 0; t < p.topk; ++t) w[t] = __fdiv_rn(w[t], ws);
  }
  for (int t = 0; t < p.topk; ++t) {
    p.sel[t] = ids[t];
    p.wts[t] = w[t];
  }
  if (p.trace_sel != nullptr) {
    const int64_t pos = p.state->pos;
    for (int t = 0; t < p.topk; ++t) {
      p.trace_sel[(pos * p.n_layers + p.layer) * p.topk + t] = ids[t];
    }
    if (p.trace_gap != nullptr) {
      p.trace_gap[pos * p.n_layers + p.layer] =
          p.topk < E ? __fsub_rn(pr[ids[p.topk - 1]], pr[ids[p.topk]]) : 1.f;
    }
  }
  *p.ticket = 0u;
}

// ------------------------------------------------------------------ gate/up
struct GateUpArgs {
  const float* h;
  const float* norm;
  float eps;
  const int32_t* wsel;
  int topk;
  const uint8_t* gate;
  const uint8_t* up;
  int tg, tu;
  uint64_t gate_nb2, up_nb2, rb_g, rb_u;
  int K, F;
  int lpr, half;  // lanes per row; output rows per job (sub-rows = 2*half)
  int jobs_per_expert, jobs_total;
  uint32_t stage_bytes, up_off;
  float* ff;
};

__device__ __forceinline__ float silu_mul(float g, float u) {
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
  return __fmul_rn(s, u);
}

__global__ void __launch_bounds__(kMoeWarps * 32) gate_up_kernel(const GateUpArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.K);
  const size_t act_bytes = (act_smem_bytes(p.K) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  uint8_t* stage = smem + act_bytes + 48 * sizeof(double);
  const bool quant = p.tg != NH_TYPE_F32;
  prep_act(a, p.h, p.norm, true, p.eps, quant, red);
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint8_t* wb = stage + static_cast<size_t>(warp) * kMoeStages * p.stage_bytes;
  const int nsb = p.K / QK;

  auto job_rows = [&](int j, int& i, int& e, int& r0, int& n) {
    i = j / p.jobs_per_expert;
    r0 = (j % p.jobs_per_expert) * p.half;
    n = min(p.half, p.F - r0);
    e = p.wsel[i];
  };
  auto issue = [&](int j, uint8_t* buf) {
    if (!quant) return;
    int i, e, r0, n;
    job_rows(j, i, e, r0, n);
    stage_bytes_warp(buf, p.gate + e * p.gate_nb2 + r0 * p.rb_g, n * p.rb_g, lane);
    stage_bytes_warp(buf + p.up_off, p.up + e * p.up_nb2 + r0 * p.rb_u, n * p.rb_u, lane);
  };
#pragma unroll
  for (int st = 0; st < kMoeStages; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) issue(j, wb + st * p.stage_bytes);
    cp_async_commit();
  }
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    cp_async_wait<kMoeStages - 1>();
    __syncwarp();
    uint8_t* buf = wb + (it % kMoeStages) * p.stage_bytes;
    int i, e, r0, n;
    job_rows(j, i, e, r0, n);
    if (quant) {
      const int sub = lane % p.lpr, kr = lane / p.lpr;
      const bool is_up = kr >= p.half;
      const int rr = is_up ? kr - p.half : kr;
      const uint8_t* src = is_up ? p.up + e * p.up_nb2 + r0 * p.rb_u : p.gate + e * p.gate_nb2 + r0 * p.rb_g;
      const uint8_t* base = (is_up ? buf + p.up_off : buf) + (reinterpret_cast<uintptr_t>(src) & 15);
      const uint64_t rb = is_up ? p.rb_u : p.rb_g;
      const int type = is_up ? p.tu : p.tg;
      const float v = row_dot_q(base + rr * rb, type, nsb, sub, p.lpr, a);
      const float u = __shfl_sync(0xffffffffu, v, (lane + p.half * p.lpr) & 31);
      if (!is_up && sub == 0 && rr < n) {
        p.ff[static_cast<int64_t>(i) * p.F + r0 + rr] = silu_mul(v, u);
      }
    } else {
      const float* grow = reinterpret_cast<const float*>(p.gate + e * p.gate_nb2 + r0 * p.rb_g);
      const float* urow = reinterpret_cast<const float*>(p.up + e * p.up_nb2 + r0 * p.rb_u);
      const float g = row_dot_f32(grow, a.xf, p.K, lane);
      const float u = row_dot_f32(urow, a.xf, p.K, lane);
      if (lane == 0) p.ff[static_cast<int64_t>(i) * p.F + r0] = silu_mul(g, u);
    }
    __syncwarp();
    const int jn = gw + (it + kMoeStages) * tw;
    if (jn < p.jobs_total) issue(jn, buf);
    cp_async_commit();
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ down + combine
struct DownArgs {
  const NhDecodeState* state;
  const float* ff;
  const int32_t* wsel;
  const float* wts;
  int topk;
  const uint8_t* down;
  int td;
  uint64_t nb2, rb;
  int F, D;
  int lpr, rows;  // lanes per row; output rows per job
  int jobs_total;
  uint32_t stage_bytes, slot_bytes;
  float* h;
  float* dump;
  int64_t dump_stride, dump_off;
};

// Q8_K quantisation of ff (topk*F values, per-256 blocks) straight from global
// memory into the activation's quant arrays.
__device__ void prep_quant_global(ActSmem& a, const float* __restrict__ src, int n) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int b = warp; b < n / QK; b += nw) {
    const float* x = src + b * QK;
    float xv[8];
    float amax = 0.f, mx = 0.f;
    int idx = INT_MAX;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      xv[k] = x[lane * 8 + k];
      const float ax = fabsf(xv[k]);
      if (ax > amax) {
        amax = ax;
        mx = xv[k];
        idx = lane * 8 + k;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (oa > amax || (oa == amax && oi < idx)) {
        amax = oa;
        mx = om;
        idx = oi;
      }
    }
    int8_t* q = a.qs + b * QK;
    if (amax == 0.f) {
#pragma unroll
      for (int k = 0; k < 8; ++k) q[lane * 8 + k] = 0;
      if (lane < 16) a.bsums[b * 16 + lane] = 0;
      if (lane == 0) a.d[b] = 0.f;
      continue;
    }
    const float iscale = __fdiv_rn(-127.f, mx);
    int part = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      int v = min(127, __float2int_rn(__fmul_rn(iscale, xv[k])));
      q[lane * 8 + k] = static_cast<int8_t>(v);
      part += v;
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    if ((lane & 1) == 0) a.bsums[b * 16 + (lane >> 1)] = static_cast<int16_t>(part);
    if (lane == 0) a.d[b] = __fdiv_rn(1.f, iscale);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kMoeWarps * 32) down_kernel(const DownArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KF = p.topk * p.F;
  const bool quant = p.td != NH_TYPE_F32;
  ActSmem a = carve_act(smem, KF);
  const size_t act_bytes = (act_smem_bytes(KF) + 15) & ~static_cast<size_t>(15);
  float* ybuf = reinterpret_cast<float*>(smem + act_bytes);  // [warps][topk][rows]
  uint8_t* stage = smem + act_bytes + static_cast<size_t>(kMoeWarps) * kMaxTopK * 32 * sizeof(float);
  if (quant) {
    prep_quant_global(a, p.ff, KF);
  } else {
    for (int i = threadIdx.x; i < KF; i += blockDim.x) a.xf[i] = p.ff[i];
    __syncthreads();
  }
  const int pos = p.state->pos, n_prompt = p.state->n_prompt;
  const bool dump = p.dump != nullptr && pos >= n_prompt - 1;
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint8_t* wb = stage + static_cast<size_t>(warp) * kMoeStages * p.stage_bytes;
  float* yw = ybuf + warp * kMaxTopK * 32;
  const int nsb = p.F / QK;
  const int rpp = 32 / p.lpr;  // sub-rows per pass

  auto issue = [&](int j, uint8_t* buf) {
    if (!quant) return;
    const int r0 = j * p.rows;
    const int n = min(p.rows, p.D - r0);
    for (int i = 0; i < p.topk; ++i) {
      stage_bytes_warp(buf + i * p.slot_bytes, p.down + p.wsel[i] * p.nb2 + r0 * p.rb, n * p.rb, lane);
    }
  };
#pragma unroll
  for (int st = 0; st < kMoeStages; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) issue(j, wb + st * p.stage_bytes);
    cp_async_commit();
  }
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    cp_async_wait<kMoeStages - 1>();
    __syncwarp();
    uint8_t* buf = wb + (it % kMoeStages) * p.stage_bytes;
    const int r0 = j * p.rows;
    const int n = min(p.rows, p.D - r0);
    if (quant) {
      // Sub-row index q enumerates (expert i, row rr): q = i*rows + rr.
      const int nq = p.topk * p.rows;
      const int sub = lane % p.lpr;
      for (int q0 = 0; q0 < nq; q0 += rpp) {
        const int q = q0 + lane / p.lpr;
        const int i = min(q / p.rows, p.topk - 1), rr = q % p.rows;
        const uint8_t* src = p.down + p.wsel[i] * p.nb2 + r0 * p.rb;
        const uint8_t* row = buf + i * p.slot_bytes + (reinterpret_cast<uintptr_t>(src) & 15) + rr * p.rb;
        ActSmem ai = a;
        ai.qs = a.qs + i * p.F;
        ai.d = a.d + i * (p.F / QK);
        ai.bsums = a.bsums + i * (p.F / 16);
        const float v = row_dot_q(row, p.td, nsb, sub, p.lpr, ai);
        if (sub == 0 && q < nq) yw[q] = v;
      }
    } else {
      for (int i = 0; i < p.topk; ++i) {
        const float* w = reinterpret_cast<const float*>(p.down + p.wsel[i] * p.nb2 + r0 * p.rb);
        const float v = row_dot_f32(w, a.xf + i * p.F, p.F, lane);
        if (lane == 0) yw[i * p.rows] = v;
      }
    }
    __syncwarp();
    if (lane < n) {
      // ggml_mul by the routing weights, then the chained adds in top-k order.
      float acc = __fmul_rn(yw[lane], p.wts[0]);
      for (int i = 1; i < p.topk; ++i) acc = __fadd_rn(acc, __fmul_rn(yw[i * p.rows + lane], p.wts[i]));
      const int r = r0 + lane;
      const float hv = __fadd_rn(p.h[r], acc);
      p.h[r] = hv;
      if (dump) p.dump[static_cast<int64_t>(pos - n_prompt + 1) * p.dump_stride + p.dump_off + r] = hv;
    }
    __syncwarp();
    const int jn = gw + (it + kMoeStages) * tw;
    if (jn < p.jobs_total) issue(jn, buf);
    cp_async_commit();
  }
  cp_async_wait<0>();
}

template <typename Kern>
bool ensure_smem(Kern k, size_t bytes, size_t& configured) {
  if (bytes <= configured) return true;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) != cudaSuccess)
    return false;
  configured = bytes;
  return true;
}

}  // namespace nh

using namespace nh;

extern "C" int64_t nh_router_scratch_bytes(int n_expert) { return 64 + 4 * static_cast<int64_t>(n_expert) + 64; }

extern "C" int nh_router_topk(const NhDecodeState* state, const float* h, const float* ffn_norm,
                              float eps, const float* router, int64_t n_embd, int n_expert, int k,
                              int norm_topk, int32_t* sel, float* wts, int32_t* trace_sel,
                              float* trace_gap, int layer, int n_layers, void* scratch,
                              void* stream) {
  if (state == nullptr || h == nullptr || router == nullptr || sel == nullptr || wts == nullptr ||
      scratch == nullptr)
    return NH_E_ARG;
  if (n_expert <= 0 || n_expert > 256 || k <= 0 || k > kMaxTopK || k > n_expert || n_embd <= 0 ||
      n_embd > kMaxK)
    return NH_E_ARG;
  RouterArgs p;
  p.state = state;
  p.h = h;
  p.norm = ffn_norm;
  p.eps = eps;
  p.router = router;
  p.K = static_cast<int>(n_embd);
  p.E = n_expert;
  p.topk = k;
  p.norm_topk = norm_topk;
  p.layer = layer;
  p.n_layers = n_layers;
  p.sel = sel;
  p.wts = wts;
  p.trace_sel = trace_sel;
  p.trace_gap = trace_gap;
  p.ticket = static_cast<unsigned*>(scratch);
  p.logits = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + 64);
  const size_t smem = act_smem_bytes(p.K);
  static size_t configured = 48 * 1024;
  if (!ensure_smem(router_kernel, smem, configured)) return NH_E_CUDA;
  const int grid = (n_expert + kRouterWarps - 1) / kRouterWarps;
  router_kernel<<<grid, kRouterWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

extern "C" int nh_moe_gate_up(const float* h, const float* ffn_norm, float eps,
                              const int32_t* wsel, int k, const void* gate, int32_t tg,
                              uint64_t gate_nb2, const void* up, int32_t tu, uint64_t up_nb2,
                              int64_t n_embd, int64_t n_ff, float* ff, void* stream) {
  if (h == nullptr || wsel == nullptr || gate == nullptr || up == nullptr || ff == nullptr) return NH_E_ARG;
  if (k <= 0 || k > kMaxTopK || n_embd <= 0 || n_embd > kMaxK || n_ff <= 0) return NH_E_ARG;
  const bool quant = tg != NH_TYPE_F32;
  if ((tg == NH_TYPE_F32) != (tu == NH_TYPE_F32)) return NH_E_TYPE;
  for (int t : {tg, tu})
    if (t != NH_TYPE_F32 && t != NH_TYPE_Q4_K && t != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (quant && n_embd % QK != 0) return NH_E_ARG;
  GateUpArgs p;
  p.h = h;
  p.norm = ffn_norm;
  p.eps = eps;
  p.wsel = wsel;
  p.topk = k;
  p.gate = static_cast<const uint8_t*>(gate);
  p.up = static_cast<const uint8_t*>(up);
  p.tg = tg;
  p.tu = tu;
  p.gate_nb2 = gate_nb2;
  p.up_nb2 = up_nb2;
  p.K = static_cast<int>(n_embd);
  p.F = static_cast<int>(n_ff);
  p.rb_g = row_bytes(tg, n_embd);
  p.rb_u = row_bytes(tu, n_embd);
  if (quant) {
    p.lpr = lanes_per_row(p.K / QK);
    if (p.lpr > 16) return NH_E_ARG;
    p.half = (32 / p.lpr) / 2;
    const uint64_t gb = (p.rb_g * p.half + 32 + 15) & ~15ull;
    const uint64_t ub = (p.rb_u * p.half + 32 + 15) & ~15ull;
    p.up_off = static_cast<uint32_t>(gb);
    p.stage_bytes = static_cast<uint32_t>(gb + ub);
  } else {
    p.lpr = 32;
    p.half = 1;
    p.up_off = 0;
    p.stage_bytes = 16;
  }
  p.jobs_per_expert = (p.F + p.half - 1) / p.half;
  p.jobs_total = p.jobs_per_expert * k;
  p.ff = ff;
  const size_t smem = ((act_smem_bytes(p.K) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double) +
                      static_cast<size_t>(kMoeWarps) * kMoeStages * p.stage_bytes;
  static size_t configured = 48 * 1024;
  if (!ensure_smem(gate_up_kernel, smem, configured)) return NH_E_CUDA;
  int grid = (p.jobs_total + kMoeWarps - 1) / kMoeWarps;
  const int cap = moe_sm_count() * (smem > 110 * 1024 ? 1 : 2);
  if (grid > cap) grid = cap;
  gate_up_kernel<<<grid, kMoeWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

extern "C" int nh_moe_down_combine(const NhDecodeState* state, const float* ff,
                                   const int32_t* wsel, const float* wts, int k, const void* down,
                                   int32_t td, uint64_t down_nb2, int64_t n_ff, int64_t n_embd,
                                   float* h_io, float* dump, int64_t dump_step_stride,
                                   int64_t dump_offset, void* stream) {
  if (state == nullptr || ff == nullptr || wsel == nullptr || wts == nullptr || down == nullptr ||
      h_io == nullptr)
    return NH_E_ARG;
  if (k <= 0 || k > kMaxTopK || n_ff <= 0 || n_embd <= 0) return NH_E_ARG;
  if (td != NH_TYPE_F32 && td != NH_TYPE_Q4_K && td != NH_TYPE_Q6_K) return NH_E_TYPE;
  const bool quant = td != NH_TYPE_F32;
  if (quant && n_ff % QK != 0) return NH_E_ARG;
  if (static_cast<int64_t>(k) * n_ff > 4 * kMaxK) return NH_E_ARG;
  DownArgs p;
  p.state = state;
  p.ff = ff;
  p.wsel = wsel;
  p.wts = wts;
  p.topk = k;
  p.down = static_cast<const uint8_t*>(down);
  p.td = td;
  p.nb2 = down_nb2;
  p.rb = row_bytes(td, n_ff);
  p.F = static_cast<int>(n_ff);
  p.D = static_cast<int>(n_embd);
  if (quant) {
    p.lpr = lanes_per_row(p.F / QK);
    const int rpp = 32 / p.lpr;
    p.rows = rpp >= k ? rpp / k : 1;
    if (p.rows > 32) p.rows = 32;
    p.slot_bytes = static_cast<uint32_t>((p.rb * p.rows + 32 + 15) & ~15ull);
    p.stage_bytes = p.slot_bytes * k;
  } else {
    p.lpr = 32;
    p.rows = 1;
    p.slot_bytes = 16;
    p.stage_bytes = 16;
  }
  if (p.rows * k > kMaxTopK * 32) return NH_E_ARG;
  p.jobs_total = (p.D + p.rows - 1) / p.rows;
  p.h = h_io;
  p.dump = dump;
  p.dump_stride = dump_step_stride;
  p.dump_off = dump_offset;
  const int KF = k * p.F;
  const size_t smem = ((act_smem_bytes(KF) + 15) & ~static_cast<size_t>(15)) +
                      static_cast<size_t>(kMoeWarps) * kMaxTopK * 32 * sizeof(float) +
                      static_cast<size_t>(kMoeWarps) * kMoeStages * p.stage_bytes;
  if (smem > 220 * 1024) return NH_E_ARG;
  static size_t configured = 48 * 1024;
  if (!ensure_smem(down_kernel, smem, configured)) return NH_E_CUDA;
  int grid = (p.jobs_total + kMoeWarps - 1) / kMoeWarps;
  const int cap = moe_sm_count() * (smem > 110 * 1024 ? 1 : 2);
  if (grid > cap) grid = cap;
  down_kernel<<<grid, kMoeWarps * 32, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

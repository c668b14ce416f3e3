// MoE kernels for one decode position: router top-k, expert gate/up with
// SwiGLU, expert down projection with the weighted top-k-order combine.
//
// Expert weights are addressed as base + wsel[i] * nb2 (+ row * row_bytes),
// so the same kernels read the resident fused expert tensors or the HBM slot
// pool of the streaming path (where wsel holds slot indices).  Both expert
// kernels stage rows with per-warp cp.async.bulk rings (rowdot.cuh); their
// weights depend on the router's choice, so staging starts after
// griddepcontrol.wait.  The gate/up kernel also prefetches the chosen
// experts' down rows into L2 for the kernel that follows it.
#include <algorithm>
#include <climits>
#include <cstring>
#include <utility>

#include "launch.cuh"
#include "attention.cuh"
#include "gemv3.cuh"
#include "rowdot3.cuh"

namespace nh {

constexpr int kMoeWarps = 8;
constexpr int kMoeMaxStages = 4;
constexpr int kRouterWarps = 8;
constexpr int kMaxTopK = 32;
constexpr int kMaxExperts = 256;

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

// f32 router row in registers: lane l holds elements 4l + 128t (t < K/128).
constexpr int kRouterMaxVec = kMaxK / 128;

// The dot of router row e with the normalised activation (xf), the row's
// lane slice already in registers when K % 128 == 0 (DotF32Vec128 order).
__device__ __forceinline__ float router_logit(const RouterArgs& p, const float4 (&wv)[kRouterMaxVec],
                                              const ActSmem& a, int e, int lane) {
  if ((p.K % 128) == 0) {
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < kRouterMaxVec; ++t) {
      if (t < p.K / 128) {
        const float4 x = *reinterpret_cast<const float4*>(a.xf + 4 * lane + 128 * t);
        s = __fadd_rn(s, __fmul_rn(wv[t].x, x.x));
        s = __fadd_rn(s, __fmul_rn(wv[t].y, x.y));
        s = __fadd_rn(s, __fmul_rn(wv[t].z, x.z));
        s = __fadd_rn(s, __fmul_rn(wv[t].w, x.w));
      }
    }
    return warp_sum(s);
  }
  return row_dot_f32(p.router + static_cast<int64_t>(e) * p.K, a.xf, p.K, lane);
}

__device__ __forceinline__ void router_load_row(const RouterArgs& p, float4 (&wv)[kRouterMaxVec], int e, int lane) {
  if ((p.K % 128) == 0 && e < p.E) {
    const float4* w4 = reinterpret_cast<const float4*>(p.router + static_cast<int64_t>(e) * p.K);
#pragma unroll
    for (int t = 0; t < kRouterMaxVec; ++t)
      if (t < p.K / 128) wv[t] = w4[lane + 32 * t];
  }
}

// Block-wide expert selection from the E router logits; any CTA that has the
// logits may run it and all obtain the same result.  Warp 0 forms
// ggml_soft_max (exp(x - max) in f32, lane l holding experts l, l+32, ...,
// summed per lane then across lanes in double, scaled by 1/sum); thread i
// then ranks expert i against all E probabilities (descending, equal
// probabilities keep the lower expert id first: the order repeated argmax
// would produce) and the top-(k+1) land in rank order.  Writes the k chosen
// experts and their weights (renormalised when norm_topk, clamped sum
// 6.103515625e-5) to o_sel/o_wts (shared) and, when `outputs`, to p.sel,
// p.wts and the trace.  Needs blockDim.x >= 32 and >= k; ends synchronised.
// `pr`: in warp 0, lane l's logits of experts l, l+32, ... (-INF beyond E).
constexpr int kLogitsPerLane = kMaxExperts / 32;  // absent experts add exact zeros to the sums

__device__ __forceinline__ void router_select_core(const RouterArgs& p, float (&pr)[kLogitsPerLane], bool outputs,
                                                   int64_t pos, int* o_sel, float* o_wts) {
  __shared__ __align__(16) float s_prob[kMaxExperts];
  __shared__ int s_ids[kMaxTopK + 1];
  __shared__ float s_vals[kMaxTopK + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.E;
  const int kk = min(p.topk + 1, E);
  // Every output slot starts in range: NaN probabilities (a corrupted
  // activation) have no strict order and their ranks may collide.
  if (tid < kk) {
    s_ids[tid] = tid;
    s_vals[tid] = 0.f;
  }
  if (warp == 0) {
    constexpr int kPer = kLogitsPerLane;
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kPer; ++k) mx = fmaxf(mx, pr[k]);
    mx = warp_max(mx);
    double sum = 0.0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = lane + 32 * k;
      pr[k] = i < E ? exp_cw(__fsub_rn(pr[k], mx)) : 0.f;
      sum += static_cast<double>(pr[k]);
    }
    sum = warp_sum_d(sum);
    const float inv = static_cast<float>(1.0 / sum);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = lane + 32 * k;
      if (i < E) s_prob[i] = __fmul_rn(pr[k], inv);
    }
  }
  __syncthreads();
  for (int i = tid; i < E; i += blockDim.x) {
    const float pi = s_prob[i];
    int r = 0;
    int j = 0;
    for (; j + 4 <= E; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(s_prob + j);
      r += (q.x > pi || (q.x == pi && j < i)) ? 1 : 0;
      r += (q.y > pi || (q.y == pi && j + 1 < i)) ? 1 : 0;
      r += (q.z > pi || (q.z == pi && j + 2 < i)) ? 1 : 0;
      r += (q.w > pi || (q.w == pi && j + 3 < i)) ? 1 : 0;
    }
    for (; j < E; ++j) r += (s_prob[j] > pi || (s_prob[j] == pi && j < i)) ? 1 : 0;
    if (r < kk) {
      s_ids[r] = i;
      s_vals[r] = pi;
    }
  }
  __syncthreads();
  if (tid < p.topk) {
    float ws = 1.f;
    if (p.norm_topk) {
      double sw = 0.0;
      for (int t = 0; t < p.topk; ++t) sw += static_cast<double>(s_vals[t]);
      ws = fmaxf(static_cast<float>(sw), 6.103515625e-5f);
    }
    const int id = s_ids[tid];
    const float w = p.norm_topk ? __fdiv_rn(s_vals[tid], ws) : s_vals[tid];
    o_sel[tid] = id;
    o_wts[tid] = w;
    if (outputs) {
      p.sel[tid] = id;
      p.wts[tid] = w;
      if (p.trace_sel != nullptr) p.trace_sel[(pos * p.n_layers + p.layer) * p.topk + tid] = id;
    }
  }
  if (outputs && p.trace_sel != nullptr && p.trace_gap != nullptr && warp == 0) {
    // Smallest gap between adjacent probabilities of the descending top-(k+1).
    float g = 1.f;
    for (int t = lane; t + 1 < kk; t += 32) g = fminf(g, __fsub_rn(s_vals[t], s_vals[t + 1]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) g = fminf(g, __shfl_xor_sync(0xffffffffu, g, o));
    if (lane == 0) p.trace_gap[pos * p.n_layers + p.layer] = g;
  }
  __syncthreads();
}

// router_select_core on logits in global memory (another CTA wrote them and
// published them before this CTA's acquire).
__device__ __forceinline__ void router_select_block(const RouterArgs& p, const float* logits, bool outputs,
                                                    int64_t pos, int* o_sel, float* o_wts) {
  float pr[kLogitsPerLane];
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kLogitsPerLane; ++k) {
    const int i = lane + 32 * k;
    pr[k] = (threadIdx.x < 32 && i < p.E) ? __ldcg(logits + i) : -INFINITY;
  }
  router_select_core(p, pr, outputs, pos, o_sel, o_wts);
}

__global__ void __launch_bounds__(kRouterWarps * 32) router_kernel(const RouterArgs p) {
  const unsigned ph_idx = phase_begin();
  extern __shared__ __align__(128) uint8_t smem[];
  ActSmem a = carve_act(smem, p.K, true, true);
  __shared__ double red[48];
  __shared__ bool s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouterWarps + warp;
  // The router weights do not depend on the preceding kernel: load the row
  // before waiting for it.
  float4 wv[kRouterMaxVec];
  router_load_row(p, wv, e, lane);
  act_load_norm(a, p.norm);
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  prep_act(a, p.h, p.norm != nullptr, true, p.eps, false, red);
  if (e < p.E) {
    const float v = router_logit(p, wv, a, e, lane);
    if (lane == 0) p.logits[e] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    if (s_last) {
      *p.ticket = 0u;  // every CTA has taken its ticket
      __threadfence();
    }
  }
  __syncthreads();
  phase_end(kPhRouter, ph_idx);
  if (!s_last) return;
  __shared__ int s_sel[kMaxTopK];
  __shared__ float s_wts[kMaxTopK];
  router_select_block(p, p.logits, true, p.state->pos, s_sel, s_wts);
}

// ------------------------------------------------------------------ gate/up
// The k selected experts (or slots): wsel in device memory, or, when wsel is
// null, the copy in wsel_inline passed with the launch.
__device__ __forceinline__ int sel_at(const int32_t* wsel, const int32_t (&inl)[kMaxTopK], int i) {
  return wsel != nullptr ? wsel[i] : inl[i];
}

struct GateUpArgs {
  NhDecodeState* state;
  const float* h;
  const float* norm;
  float eps;
  const int32_t* wsel;
  int32_t wsel_inline[kMaxTopK];
  int topk;
  const uint8_t* gate;
  const uint8_t* up;
  int tg, tu;
  uint64_t gate_nb2, up_nb2, rb_g, rb_u;
  int K, F;
  int lpr, rpp;   // lanes per row, rows per pass
  int R;          // output rows per job (R gate rows + R up rows)
  int S;          // ring depth (<= kMoeMaxStages)
  int jobs_per_expert, jobs_total;
  uint32_t stage_bytes, up_off;
  float* ff;
  // L2 prefetch of the down rows of the chosen experts
  const uint8_t* down;
  uint64_t down_nb2;
};

__device__ __forceinline__ float silu_mul(float g, float u) {
  const float s = __fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g)));
  return __fmul_rn(s, u);
}

template <int CPL>
__global__ void __launch_bounds__(kMoeWarps * 32) gate_up_kernel(const GateUpArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool quant = p.tg != NH_TYPE_F32;
  ActSmem a = carve_act(smem, p.K, true, true);
  const size_t act_bytes = (act_smem_bytes(p.K, true, true) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  float* ybuf = reinterpret_cast<float*>(smem + act_bytes + 48 * sizeof(double));  // [warps][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes + 48 * sizeof(double) + kMoeWarps * 64 * sizeof(float));
  uint8_t* stage = reinterpret_cast<uint8_t*>(bars + kMoeWarps * p.S);
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  float* yw = ybuf + warp * 64;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  act_load_norm(a, p.norm);
  pdl_wait();
  pdl_trigger();

  auto job_rows = [&](int j, int& i, int& e, int& r0, int& n) {
    i = j / p.jobs_per_expert;
    r0 = (j % p.jobs_per_expert) * p.R;
    n = min(p.R, p.F - r0);
    e = sel_at(p.wsel, p.wsel_inline, i);
  };
  auto issue = [&](int j, int st) {
    if (!quant || lane != 0) return;
    int i, e, r0, n;
    job_rows(j, i, e, r0, n);
    uint32_t lg, og, lu, ou;
    const uint8_t* sg = span16(p.gate + e * p.gate_nb2 + r0 * p.rb_g, n * p.rb_g, &lg, &og);
    const uint8_t* su = span16(p.up + e * p.up_nb2 + r0 * p.rb_u, n * p.rb_u, &lu, &ou);
    mbar_expect_tx(&wbar[st], lg + lu);
    uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
    bulk_g2s(buf, sg, lg, &wbar[st]);
    bulk_g2s(buf + p.up_off, su, lu, &wbar[st]);
  };
#pragma unroll
  for (int st = 0; st < p.S; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) issue(j, st);
  }
  // Warm L2 with this layer's chosen down rows for the next kernel.
  if (p.down != nullptr && threadIdx.x < p.topk) {
    const int e = sel_at(p.wsel, p.wsel_inline, threadIdx.x);
    const uint64_t per = p.down_nb2 / gridDim.x;
    const uint64_t beg = (per * blockIdx.x) & ~static_cast<uint64_t>(15);
    const uint64_t end = blockIdx.x + 1 == gridDim.x ? p.down_nb2 : ((per * (blockIdx.x + 1)) & ~static_cast<uint64_t>(15));
    if (end > beg) prefetch_l2(p.down + e * p.down_nb2 + beg, static_cast<uint32_t>(end - beg));
  }
  prep_act(a, p.h, p.norm != nullptr, true, p.eps, quant, red);
  const int jl = lane % p.lpr, kr = lane / p.lpr;
  ActReg<CPL> ar;
  if (quant) load_act<CPL>(ar, a, 0, jl, p.lpr);
  bool failed = false;
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    const int st = it % p.S;
    int i, e, r0, n;
    job_rows(j, i, e, r0, n);
    if (quant) {
      if (!mbar_wait(&wbar[st], (it / p.S) & 1)) {
        failed = true;
        break;
      }
      const uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
      const uint32_t og = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.gate + e * p.gate_nb2 + r0 * p.rb_g) & 15);
      const uint32_t ou = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.up + e * p.up_nb2 + r0 * p.rb_u) & 15);
      // Sub-row u < R: gate row r0+u; R <= u < 2R: up row r0+u-R.
      for (int u0 = 0; u0 < 2 * p.R; u0 += p.rpp) {
        const int u = u0 + kr;
        const bool is_up = u >= p.R;
        const int rr = is_up ? u - p.R : u;
        const uint8_t* row = is_up ? buf + p.up_off + ou + rr * p.rb_u : buf + og + rr * p.rb_g;
        const float v = row_dot_reg<CPL>(row, is_up ? p.tu : p.tg, jl, p.lpr, ar);
        if (jl == 0 && u < 2 * p.R) yw[u] = v;
      }
      __syncwarp();
      if (lane < n) p.ff[static_cast<int64_t>(i) * p.F + r0 + lane] = silu_mul(yw[lane], yw[p.R + lane]);
    } else {
      const float* grow = reinterpret_cast<const float*>(p.gate + e * p.gate_nb2 + r0 * p.rb_g);
      const float* urow = reinterpret_cast<const float*>(p.up + e * p.up_nb2 + r0 * p.rb_u);
      const float g = row_dot_f32(grow, a.xf, p.K, lane);
      const float u = row_dot_f32(urow, a.xf, p.K, lane);
      if (lane == 0) p.ff[static_cast<int64_t>(i) * p.F + r0] = silu_mul(g, u);
    }
    __syncwarp();
    const int jn = gw + (it + p.S) * tw;
    if (jn < p.jobs_total) issue(jn, st);
  }
  if (failed && lane == 0 && p.state != nullptr) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
}

// ------------------------------------------------------------------ down + combine
struct DownArgs {
  NhDecodeState* state;
  const float* ff;
  const int32_t* wsel;
  int32_t wsel_inline[kMaxTopK];
  const float* wts;
  int topk;
  const uint8_t* down;
  int td;
  uint64_t nb2, rb;
  int F, D;
  int lpr, rpp;  // lanes per row; rows per pass
  int R;         // output rows per job
  int S;         // ring depth (<= kMoeMaxStages)
  int ystride;   // per-warp floats of sub-row results (>= topk*R)
  int jobs_total;
  uint32_t stage_bytes, slot_bytes;
  float* h;
  float* dump;
  int64_t dump_stride, dump_off;
};

template <int CPL>
__global__ void __launch_bounds__(kMoeWarps * 32) down_kernel(const DownArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KF = p.topk * p.F;
  const bool quant = p.td != NH_TYPE_F32;
  ActSmem a = carve_act(smem, KF, !quant);
  const size_t act_bytes = (act_smem_bytes(KF, !quant) + 15) & ~static_cast<size_t>(15);
  float* ybuf = reinterpret_cast<float*>(smem + act_bytes);  // [warps][kMaxTopK*32]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes + kMoeWarps * p.ystride * sizeof(float));
  uint8_t* stage = reinterpret_cast<uint8_t*>(bars + kMoeWarps * p.S);
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  float* yw = ybuf + warp * p.ystride;
  const int nsb = p.F / QK;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_trigger();

  auto issue = [&](int j, int st) {
    if (!quant || lane != 0) return;
    const int r0 = j * p.R;
    const int n = min(p.R, p.D - r0);
    uint32_t total = 0;
    uint32_t lens[kMaxTopK];
    const uint8_t* srcs[kMaxTopK];
    for (int i = 0; i < p.topk; ++i) {
      uint32_t off;
      srcs[i] = span16(p.down + sel_at(p.wsel, p.wsel_inline, i) * p.nb2 + r0 * p.rb, n * p.rb, &lens[i], &off);
      total += lens[i];
    }
    mbar_expect_tx(&wbar[st], total);
    uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
    for (int i = 0; i < p.topk; ++i) bulk_g2s(buf + i * p.slot_bytes, srcs[i], lens[i], &wbar[st]);
  };
#pragma unroll
  for (int st = 0; st < p.S; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) issue(j, st);
  }
  // The activation: each expert's ff row, Q8_K-quantised per 256-block.  A
  // warp issues the loads of up to kU blocks before quantising any of them.
  if (quant) {
    constexpr int kU = 8;
    const int nb = KF / QK;
    const bool al = (reinterpret_cast<uintptr_t>(p.ff) & 15) == 0;
    for (int b0 = warp; b0 < nb; b0 += kU * kMoeWarps) {
      float4 buf[kU][2];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int b = b0 + u * kMoeWarps;
        if (b < nb) {
          const float* src = p.ff + b * QK + lane * 8;
          if (al) {
            buf[u][0] = *reinterpret_cast<const float4*>(src);
            buf[u][1] = *reinterpret_cast<const float4*>(src + 4);
          } else {
            buf[u][0] = make_float4(src[0], src[1], src[2], src[3]);
            buf[u][1] = make_float4(src[4], src[5], src[6], src[7]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int b = b0 + u * kMoeWarps;
        if (b < nb) {
          const float v[8] = {buf[u][0].x, buf[u][0].y, buf[u][0].z, buf[u][0].w,
                              buf[u][1].x, buf[u][1].y, buf[u][1].z, buf[u][1].w};
          quantize_block_warp(v, b, a, lane);
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < KF; i += blockDim.x) a.xf[i] = p.ff[i];
  }
  __syncthreads();
  const int pos = p.state->pos, n_prompt = p.state->n_prompt;
  const bool dump = p.dump != nullptr && pos >= n_prompt - 1;
  const int jl = lane % p.lpr, kr = lane / p.lpr;
  bool failed = false;
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    const int st = it % p.S;
    const int r0 = j * p.R;
    const int n = min(p.R, p.D - r0);
    if (quant) {
      if (!mbar_wait(&wbar[st], (it / p.S) & 1)) {
        failed = true;
        break;
      }
      const uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
      // Sub-row q enumerates (expert i, row rr): q = i*R + rr.
      const int nq = p.topk * p.R;
      for (int q0 = 0; q0 < nq; q0 += p.rpp) {
        const int q = q0 + kr;
        const int i = min(q / p.R, p.topk - 1), rr = q % p.R;
        const uint32_t off =
            static_cast<uint32_t>(
                reinterpret_cast<uintptr_t>(p.down + sel_at(p.wsel, p.wsel_inline, i) * p.nb2 + r0 * p.rb) & 15);
        ActReg<CPL> ar;
        load_act<CPL>(ar, a, i * nsb, jl, p.lpr);
        const float v = row_dot_reg<CPL>(buf + i * p.slot_bytes + off + rr * p.rb, p.td, jl, p.lpr, ar);
        if (jl == 0 && q < nq) yw[q] = v;
      }
    } else {
      for (int i = 0; i < p.topk; ++i) {
        const float* w = reinterpret_cast<const float*>(p.down + sel_at(p.wsel, p.wsel_inline, i) * p.nb2 + r0 * p.rb);
        const float v = row_dot_f32(w, a.xf + i * p.F, p.F, lane);
        if (lane == 0) yw[i * p.R] = v;
      }
    }
    __syncwarp();
    if (lane < n) {
      // ggml_mul by the routing weights, then the chained adds in top-k order.
      float acc = __fmul_rn(yw[lane], p.wts[0]);
      for (int i = 1; i < p.topk; ++i) acc = __fadd_rn(acc, __fmul_rn(yw[i * p.R + lane], p.wts[i]));
      const int r = r0 + lane;
      const float hv = __fadd_rn(p.h[r], acc);
      p.h[r] = hv;
      if (dump) p.dump[static_cast<int64_t>(pos - n_prompt + 1) * p.dump_stride + p.dump_off + r] = hv;
    }
    __syncwarp();
    const int jn = gw + (it + p.S) * tw;
    if (jn < p.jobs_total) issue(jn, st);
  }
  if (failed && lane == 0) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
}

// ------------------------------------------------------------------ lane-per-super-block forms
// gate/up: a job is P = 32/G rows of one expert; pass 1 computes the P gate
// rows, pass 2 the P up rows, so the lane that holds a gate row's value also
// holds the matching up row's value and writes silu(gate)*up itself.
// Job j of the gate/up kernels: expert slot i, its expert (or slot) e, the
// first output row r0 and the row count n.
__device__ __forceinline__ void gu3_job(const GateUpArgs& p, const int* s_sel, int j, int& i, int& e, int& r0,
                                        int& n) {
  i = j / p.jobs_per_expert;
  r0 = (j - i * p.jobs_per_expert) * p.rpp;
  n = min(p.rpp, p.F - r0);
  e = s_sel[i];
}

// Lane 0 stages job j's gate and up rows into stage st.
__device__ __forceinline__ void gu3_issue(const GateUpArgs& p, const int* s_sel, uint64_t* wbar, uint8_t* wb, int j,
                                          int st, int lane) {
  if (lane != 0) return;
  int i, e, r0, n;
  gu3_job(p, s_sel, j, i, e, r0, n);
  uint32_t lg, og, lu, ou;
  const uint8_t* sg = span16(p.gate + e * p.gate_nb2 + r0 * p.rb_g, n * p.rb_g, &lg, &og);
  const uint8_t* su = span16(p.up + e * p.up_nb2 + r0 * p.rb_u, n * p.rb_u, &lu, &ou);
  mbar_expect_tx(&wbar[st], lg + lu);
  uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
  bulk_g2s(buf, sg, lg, &wbar[st]);
  bulk_g2s(buf + p.up_off, su, lu, &wbar[st]);
}

// Starts the selected experts' down weights towards L2 for the down pass:
// this CTA's share, in pieces of at most 64 KB over warp 0's lanes.
__device__ __forceinline__ void gu3_prefetch_down(const GateUpArgs& p, const int* s_sel, int warp, int lane) {
  if (p.down == nullptr || warp != 0) return;
  constexpr uint64_t kPiece = 64 * 1024;
  const uint64_t total = p.down_nb2 * static_cast<uint64_t>(p.topk);
  const uint64_t share = ((total / gridDim.x) + 15) & ~static_cast<uint64_t>(15);
  const uint64_t beg = share * blockIdx.x;
  const uint64_t end = beg + share < total ? beg + share : total;
  for (uint64_t o = beg + static_cast<uint64_t>(lane) * kPiece; o < end; o += 32 * kPiece) {
    // Pieces never straddle two experts: clip at the expert boundary.
    const uint64_t i = o / p.down_nb2, in = o - i * p.down_nb2;
    uint64_t len = end - o < kPiece ? end - o : kPiece;
    if (in + len > p.down_nb2) len = p.down_nb2 - in;
    prefetch_l2(p.down + static_cast<uint64_t>(s_sel[i]) * p.down_nb2 + in, static_cast<uint32_t>(len));
  }
}

// The warp's jobs gw, gw+tw, ... (the first S already issued): returns false
// when a stage wait expired.
template <class View>
__device__ __forceinline__ bool gu3_run(const GateUpArgs& p, const int* s_sel, uint64_t* wbar, uint8_t* wb,
                                        const View& act, int gw, int tw, int lane) {
  const int G = p.lpr;
  const int g = lane % G, r = lane / G;
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    const int st = it % p.S;
    int i, e, r0, n;
    gu3_job(p, s_sel, j, i, e, r0, n);
    if (!mbar_wait(&wbar[st], (it / p.S) & 1)) return false;
    if (it == 0) phase_stamp(10);
    const uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
    const uint32_t og = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.gate + e * p.gate_nb2 + r0 * p.rb_g) & 15);
    const uint32_t ou = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.up + e * p.up_nb2 + r0 * p.rb_u) & 15);
    // Gate then up through one call site: a single copy of each dot body in
    // the code (the warps run it once or twice, so instruction fetch, not
    // issue, is what its size costs).
    float vg = 0.f, vu = 0.f;
#pragma unroll 1
    for (int w = 0; w < 2; ++w) {
      const float v = row_dot3v(w == 0 ? buf + og + r * p.rb_g : buf + p.up_off + ou + r * p.rb_u,
                                w == 0 ? p.tg : p.tu, g, G, act);
      if (w == 0)
        vg = v;
      else
        vu = v;
    }
    if (g == 0 && r < n) p.ff[static_cast<int64_t>(i) * p.F + r0 + r] = silu_mul(vg, vu);
    __syncwarp();
    const int jn = gw + (it + p.S) * tw;
    if (jn < p.jobs_total) gu3_issue(p, s_sel, wbar, wb, jn, st, lane);
  }
  return true;
}

__global__ void __launch_bounds__(kMoeWarps * 32, 2) gate_up3_kernel(const GateUpArgs p) {
  const unsigned ph_idx = phase_begin();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.K, true, true);
  const size_t act_bytes = (act_smem_bytes(p.K, true, true) + 15) & ~static_cast<size_t>(15);
  double* red = reinterpret_cast<double*>(smem + act_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes + 48 * sizeof(double));
  uint8_t* stage = reinterpret_cast<uint8_t*>(bars + kMoeWarps * p.S);
  __shared__ int s_sel[kMaxTopK];
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  act_load_norm(a, p.norm);
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  // The selection is read once; every job then finds its expert in shared memory.
  if (threadIdx.x < p.topk) s_sel[threadIdx.x] = sel_at(p.wsel, p.wsel_inline, threadIdx.x);
  __syncthreads();
  for (int st = 0; st < p.S; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) gu3_issue(p, s_sel, wbar, wb, j, st, lane);
  }
  gu3_prefetch_down(p, s_sel, warp, lane);
  prep_act(a, p.h, p.norm != nullptr, true, p.eps, true, red);
  const bool ok = gu3_run(p, s_sel, wbar, wb, Act3Smem{a, lane % p.lpr}, gw, tw, lane);
  if (!ok && lane == 0 && p.state != nullptr) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  phase_end(kPhGateUp, ph_idx);
}

// down + combine: G = F/256 lanes per row and P = 32/G row groups per pass;
// group q takes expert q % k and row q / k of the job's Rp = P/k rows, so a
// lane's activation (its expert's super-block g of ff) never changes.  The k
// values of a row are gathered by shuffles and summed in top-k order.
// Lane i < k stages expert i's rows of job j; lane 0 registers the total
// bytes on the stage's barrier before any copy is issued.  Warp-collective.
__device__ __forceinline__ void dn3_issue(const DownArgs& p, const int* s_sel, uint64_t* wbar, uint8_t* wb, int j,
                                          int st, int lane) {
  const int r0 = j * p.R;
  const int n = min(p.R, p.D - r0);
  uint32_t len = 0, off;
  const uint8_t* src = nullptr;
  if (lane < p.topk) src = span16(p.down + s_sel[lane] * p.nb2 + r0 * p.rb, n * p.rb, &len, &off);
  uint32_t total = len;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  if (lane == 0) mbar_expect_tx(&wbar[st], total);
  __syncwarp();
  if (lane < p.topk)
    bulk_g2s(wb + static_cast<size_t>(st) * p.stage_bytes + lane * p.slot_bytes, src, len, &wbar[st]);
}

// The warp's down jobs (the first S already issued) against the prepared ff
// activation: returns false when a stage wait expired.
// pos / n_prompt: the decode cursor (for the dump).  h0: when have_h0, this
// lane's h value for the warp's first job (read ahead by the caller).
__device__ __forceinline__ bool dn3_run(const DownArgs& p, const int* s_sel, const float* s_wts, uint64_t* wbar,
                                        uint8_t* wb, const ActSmem& a, int gw, int tw, int lane, int pos,
                                        int n_prompt, bool have_h0, float h0) {
  const int G = p.lpr, k = p.topk, Rp = p.R;
  const int g = lane % G, q = lane / G;
  const int ie = q % k, rr = q / k;  // this lane's expert and row within the job
  const Act3Smem act{a, ie * G + g};
  const bool dump = p.dump != nullptr && pos >= n_prompt - 1;
  const int rl = lane % Rp;  // the row this lane combines (lanes < n write it)
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    const int st = it % p.S;
    const int r0 = j * Rp;
    const int n = min(Rp, p.D - r0);
    if (!mbar_wait(&wbar[st], (it / p.S) & 1)) return false;
    if (it == 0) phase_stamp(8);
    const uint8_t* buf = wb + static_cast<size_t>(st) * p.stage_bytes;
    const uint32_t off =
        static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.down + s_sel[ie] * p.nb2 + r0 * p.rb) & 15);
    const float v = row_dot3v(buf + ie * p.slot_bytes + off + rr * p.rb, p.td, g, G, act);
    // ggml_mul by the routing weights, then the chained adds in top-k order.
    float acc = __fmul_rn(__shfl_sync(0xffffffffu, v, (rl * k) * G), s_wts[0]);
    for (int i = 1; i < k; ++i) acc = __fadd_rn(acc, __fmul_rn(__shfl_sync(0xffffffffu, v, (rl * k + i) * G), s_wts[i]));
    if (lane < n) {
      const int row = r0 + lane;
      const float hv = __fadd_rn(it == 0 && have_h0 ? h0 : __ldcg(p.h + row), acc);
      p.h[row] = hv;
      if (dump) p.dump[static_cast<int64_t>(pos - n_prompt + 1) * p.dump_stride + p.dump_off + row] = hv;
    }
    __syncwarp();
    const int jn = gw + (it + p.S) * tw;
    if (jn < p.jobs_total) dn3_issue(p, s_sel, wbar, wb, jn, st, lane);
  }
  return true;
}

__global__ void __launch_bounds__(kMoeWarps * 32, 2) down3_kernel(const DownArgs p) {
  const unsigned ph_idx = phase_begin();
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KF = p.topk * p.F;
  ActSmem a = carve_act(smem, KF, true);
  const size_t act_bytes = (act_smem_bytes(KF, true) + 15) & ~static_cast<size_t>(15);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_bytes);
  uint8_t* stage = reinterpret_cast<uint8_t*>(bars + kMoeWarps * p.S);
  __shared__ int s_sel[kMaxTopK];
  __shared__ float s_wts[kMaxTopK];
  __shared__ double red[40];
  const int gw = blockIdx.x * kMoeWarps + warp, tw = gridDim.x * kMoeWarps;
  uint64_t* wbar = bars + warp * p.S;
  uint8_t* wb = stage + static_cast<size_t>(warp) * p.S * p.stage_bytes;
  if (lane == 0) {
    for (int s = 0; s < p.S; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  if (threadIdx.x < p.topk) {
    s_sel[threadIdx.x] = sel_at(p.wsel, p.wsel_inline, threadIdx.x);
    s_wts[threadIdx.x] = p.wts[threadIdx.x];
  }
  __syncthreads();
  for (int st = 0; st < p.S; ++st) {
    const int j = gw + st * tw;
    if (j < p.jobs_total) dn3_issue(p, s_sel, wbar, wb, j, st, lane);
  }
  // The activation: the k experts' ff rows, Q8_K-quantised per 256-block.
  prep_act(a, p.ff, false, false, 0.f, true, red);
  const bool ok = dn3_run(p, s_sel, s_wts, wbar, wb, a, gw, tw, lane, p.state->pos, p.state->n_prompt, false, 0.f);
  if (!ok && lane == 0) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  phase_end(kPhDown, ph_idx);
}

// ------------------------------------------------------------------ fused layer
// Router, gate/up and down of one layer in one cooperative grid (every CTA
// resident at once).  The first router_ctas CTAs compute the logits (one warp
// per expert, the f32 row staged in shared memory before the preceding kernel
// ends) and publish each as one 64-bit word tagged with the launch (`epoch`
// + 1); every CTA polls the E words until all carry this launch's tag,
// selects the experts itself (CTA 0 also writes the router outputs), streams its
// warps' gate/up jobs and, as soon as a warp's last one is consumed, stages
// the warp's first down jobs in the same shared-memory region, so the down
// rows load while the grid gathers at sync[1] behind the last ff row.
// sync[2] counts exits; the last CTA to leave zeroes the counters and
// advances the epoch for the next launch.  Every wait is bounded and records
// NH_E_TIMEOUT.
struct FusedArgs {
  RouterArgs r;
  GateUpArgs g;
  DownArgs d;
  unsigned long long* tagged;  // [E] logits published as (tag << 32) | f32 bits
  unsigned* epoch;             // launches completed; this launch's tag is epoch + 1
  unsigned* sync;
  int router_ctas;
  uint32_t act_bytes;     // the shared activation region (gate/up, then down)
  uint32_t region_bytes;  // per-warp staging shared by the two rings
};

constexpr int kGridSpins = 1 << 24;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kLogitSpins = 1 << 21;

// Warp 0: the E logits this launch published (each a single 64-bit word
// carrying its launch tag, so a word is either this launch's value or is
// rejected), lane l getting experts l, l+32, ... (-INF beyond E).  Bounded:
// returns false if they have not all arrived after kLogitSpins polls.
__device__ __forceinline__ bool collect_logits(const unsigned long long* tagged, int E, unsigned tag, int lane,
                                               float (&pr)[kLogitsPerLane]) {
  for (int it = 0; it < kLogitSpins; ++it) {
    bool mine = true;
#pragma unroll
    for (int k = 0; k < kLogitsPerLane; ++k) {
      const int i = lane + 32 * k;
      pr[k] = -INFINITY;
      if (i < E) {
        const unsigned long long v = ld_relaxed_u64(tagged + i);
        if (static_cast<unsigned>(v >> 32) == tag)
          pr[k] = __uint_as_float(static_cast<unsigned>(v));
        else
          mine = false;
      }
    }
    if (__all_sync(0xffffffffu, mine)) return true;
  }
  return false;
}

// Adds to a grid counter with release semantics: this CTA's earlier writes
// (ordered before the calling thread by a CTA barrier) are visible to any
// thread that acquires the new count.
__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait (one thread) until *p >= target.
__device__ __forceinline__ bool wait_count(const unsigned* p, unsigned target) {
  for (int i = 0; i < kGridSpins; ++i) {
    if (ld_acquire_gpu(p) >= target) return true;
    __nanosleep(32);
  }
  return false;
}

// Q8_K quantisation of n_blocks 256-value blocks read from global memory
// (written by other CTAs of this grid: loaded through L2), each warp its
// blocks; the same per-block arithmetic as prep_act.
__device__ __forceinline__ void quant_act_global(ActSmem& a, const float* src, int n_blocks) {
  constexpr int kAhead = 4;  // blocks per warp whose loads are all in flight at once
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int b0 = warp; b0 < n_blocks; b0 += kAhead * nw) {
    float v[kAhead][8];
    int blk[kAhead];
    bool live[kAhead];
#pragma unroll
    for (int i = 0; i < kAhead; ++i) {
      blk[i] = b0 + i * nw;
      live[i] = blk[i] < n_blocks;
      float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
      if (live[i]) {
        const float4* s4 = reinterpret_cast<const float4*>(src + blk[i] * QK + lane * 8);
        lo = __ldcg(s4);
        hi = __ldcg(s4 + 1);
      }
      v[i][0] = lo.x, v[i][1] = lo.y, v[i][2] = lo.z, v[i][3] = lo.w;
      v[i][4] = hi.x, v[i][5] = hi.y, v[i][6] = hi.z, v[i][7] = hi.w;
    }
    quantize_blocks_warp<kAhead>(v, blk, live, a, lane);
  }
}

// Per-warp shared-memory handles of the MoE block: the gate/up and down ring
// barriers, the router-row barrier and the warp's staging region.
struct MoeWarp {
  uint64_t* gbar;
  uint64_t* dbar;
  uint64_t* rbar;
  uint8_t* wb;
};

struct MoeShared {
  int sel[kMaxTopK];
  float wts[kMaxTopK];
  int ok, pos, np;
  unsigned tag;
};

// Lane 0: initialise the warp's MoE barriers (the caller fences the inits).
__device__ __forceinline__ void moe_init_warp(const FusedArgs& p, const MoeWarp& w) {
  for (int s = 0; s < p.g.S; ++s) mbar_init(&w.gbar[s], 1);
  for (int s = 0; s < p.d.S; ++s) mbar_init(&w.dbar[s], 1);
  mbar_init(w.rbar, 1);
}

// Lane 0 of the router warp for expert e: stage its f32 row in the warp's
// region (free until the selection is known).
__device__ __forceinline__ void moe_stage_router_row(const FusedArgs& p, const MoeWarp& w, int e) {
  const uint32_t bytes = static_cast<uint32_t>(p.r.K) * 4u;
  mbar_expect_tx(w.rbar, bytes);
  bulk_g2s(w.wb, p.r.router + static_cast<int64_t>(e) * p.r.K, bytes, w.rbar);
}

// The MoE block of one layer once h is final, block-wide: the normalised,
// quantised activation; the router warps' logits (router_e >= 0: this warp's
// expert, its row staged by moe_stage_router_row), published tagged with
// sh.tag; the selection in every CTA once it has collected all E logits (CTA
// 0 writes the router outputs); the gate/up jobs,
// then the down rows staged in the same regions; the grid barrier sync[1];
// the ff activation and the down jobs.  The norm weight must already be in
// a.wf (act_load_norm) and sh.pos / sh.np / sh.tag set before the call.  Returns false
// where a bounded wait expired.
__device__ __forceinline__ bool moe_run(const FusedArgs& p, uint8_t* smem, const MoeWarp& w, bool router_cta,
                                        int router_e, MoeShared& sh, double* red) {
  const int lane = threadIdx.x & 31;
  const GateUpArgs& g = p.g;
  const DownArgs& d = p.d;
  ActSmem a = carve_act(smem, g.K, true, true);
  const int gw = blockIdx.x * kMoeWarps + (threadIdx.x >> 5), tw = gridDim.x * kMoeWarps;
  // The normalised f32 row first: the router reads it; its Q8_K form (for
  // gate/up only) is made while the logits travel between CTAs.
  prep_act<true>(a, g.h, g.norm != nullptr, true, g.eps, false, red);
  phase_stamp(2);
  bool ok = true;
  if (router_cta) {
    if (router_e >= 0) {
      ok = mbar_wait(w.rbar, 0);
      // DotF32Vec128 order: lane l sums elements 4l + 128t (t ascending),
      // then the butterfly across lanes.
      const float4* w4 = reinterpret_cast<const float4*>(w.wb);
      float sdot = 0.f;
      for (int t = 0; t < p.r.K / 128; ++t) {
        const float4 wv = w4[lane + 32 * t];
        const float4 x = *reinterpret_cast<const float4*>(a.xf + 4 * lane + 128 * t);
        sdot = __fadd_rn(sdot, __fmul_rn(wv.x, x.x));
        sdot = __fadd_rn(sdot, __fmul_rn(wv.y, x.y));
        sdot = __fadd_rn(sdot, __fmul_rn(wv.z, x.z));
        sdot = __fadd_rn(sdot, __fmul_rn(wv.w, x.w));
      }
      sdot = warp_sum(sdot);
      if (lane == 0)
        st_relaxed_u64(p.tagged + router_e,
                       (static_cast<unsigned long long>(sh.tag) << 32) | __float_as_uint(sdot));
    }
  }
  quant_act_smem(a);
  // Every CTA collects the logits itself (warp 0) and selects.
  float pr[kLogitsPerLane];
  if (threadIdx.x < 32) {
    const bool got = collect_logits(p.tagged, p.r.E, sh.tag, lane, pr);
    if (lane == 0) sh.ok = got;
  }
  __syncthreads();
  phase_stamp(3);
  const bool sel_ok = sh.ok != 0;
  if (sel_ok) {
    router_select_core(p.r, pr, blockIdx.x == 0, sh.pos, sh.sel, sh.wts);
    for (int st = 0; st < g.S; ++st) {
      const int j = gw + st * tw;
      if (j < g.jobs_total) gu3_issue(g, sh.sel, w.gbar, w.wb, j, st, lane);
    }
    ok = gu3_run(g, sh.sel, w.gbar, w.wb, Act3Smem{a, lane % g.lpr}, gw, tw, lane) && ok;
    phase_stamp(4);
    if (ok) {
      for (int st = 0; st < d.S; ++st) {
        const int j = gw + st * tw;
        if (j < d.jobs_total) dn3_issue(d, sh.sel, w.dbar, w.wb, j, st, lane);
      }
    }
  }
  // The residual rows of this warp's first down job (only this warp writes
  // them), read ahead of the grid barrier.
  float h0 = 0.f;
  if (gw < d.jobs_total && lane < min(d.R, d.D - gw * d.R)) h0 = __ldcg(d.h + gw * d.R + lane);
  // Grid barrier: every ff row written before any CTA quantises ff.  Launches
  // alternate between two arrival counters by the parity of their tag; CTA 0
  // zeroed this launch's counter at the start of the previous launch.
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* arrived = &p.sync[1 + (sh.tag & 1u)];
    red_release_gpu(arrived, 1u);
    sh.ok = wait_count(arrived, gridDim.x);
    // Every CTA read the epoch before arriving: CTA 0 advances it.
    if (blockIdx.x == 0) *p.epoch = sh.tag;
  }
  __syncthreads();
  phase_stamp(5);
  bool ok_dn = ok && sel_ok && sh.ok != 0;
  if (sh.ok != 0 && sel_ok) {
    // The gate/up activation is no longer read: the ff activation takes its place.
    ActSmem af = carve_act(smem, d.topk * d.F, false);
    quant_act_global(af, d.ff, d.topk * d.F / QK);
    __syncthreads();
    phase_stamp(6);
    if (ok_dn) ok_dn = dn3_run(d, sh.sel, sh.wts, w.dbar, w.wb, af, gw, tw, lane, sh.pos, sh.np, true, h0);
  }
  return ok_dn;
}

__device__ __forceinline__ MoeWarp moe_warp(const FusedArgs& p, uint8_t* smem, int warp, int extra_bars) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.act_bytes + 48 * sizeof(double));
  MoeWarp w;
  w.gbar = bars + warp * p.g.S;
  w.dbar = bars + kMoeWarps * p.g.S + warp * p.d.S;
  w.rbar = bars + kMoeWarps * (p.g.S + p.d.S) + warp;
  w.wb = reinterpret_cast<uint8_t*>(bars + kMoeWarps * (p.g.S + p.d.S + 1 + extra_bars)) +
         static_cast<size_t>(warp) * p.region_bytes;
  return w;
}

// One function serves every weight-type mix (types are dispatched at run
// time): a single copy of its code stays warm in the instruction caches from
// layer to layer, which measured faster than per-type variants.
__global__ void __launch_bounds__(kMoeWarps * 32, 2) moe_fused_kernel(const __grid_constant__ FusedArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const unsigned ph_idx = phase_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ActSmem a = carve_act(smem, p.g.K, true, true);
  double* red = reinterpret_cast<double*>(smem + p.act_bytes);
  const MoeWarp w = moe_warp(p, smem, warp, 0);
  __shared__ MoeShared sh;
  const bool router_cta = static_cast<int>(blockIdx.x) < p.router_ctas;
  const int e = blockIdx.x * kMoeWarps + warp;
  const int router_e = router_cta && e < p.r.E ? e : -1;
  if (lane == 0) {
    moe_init_warp(p, w);
    fence_barrier_init();
    if (router_e >= 0) moe_stage_router_row(p, w, router_e);
  }
  act_load_norm(a, p.g.norm);
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  if (threadIdx.x == 0) {
    sh.pos = p.d.state->pos;
    sh.np = p.d.state->n_prompt;
    sh.tag = *reinterpret_cast<volatile unsigned*>(p.epoch) + 1u;
    // The other arrival counter was last used by the previous launch, which
    // has completed; the next launch uses it.
    if (blockIdx.x == 0) p.sync[1 + ((sh.tag + 1u) & 1u)] = 0u;
  }
  const bool ok = moe_run(p, smem, w, router_cta, router_e, sh, red);
  phase_stamp(7);
  phase_end_sync(kPhMoeFused, ph_idx);
  if (!ok && lane == 0) atomicCAS(&p.d.state->error, 0, NH_E_TIMEOUT);
}

}  // namespace nh

using namespace nh;

namespace {
int launch_router(const RouterArgs& p, size_t smem, int grid, cudaStream_t st) {
  static SmemLimit configured;
  if (!ensure_smem(router_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(router_kernel, dim3(grid), dim3(kRouterWarps * 32), smem, st, p);
}
}  // namespace

extern "C" int64_t nh_router_scratch_bytes(int n_expert) { return 64 + 4 * static_cast<int64_t>(n_expert) + 64; }

extern "C" int nh_router_topk(const NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                              const float* router, int64_t n_embd, int n_expert, int k, int norm_topk, int32_t* sel,
                              float* wts, int32_t* trace_sel, float* trace_gap, int layer, int n_layers,
                              void* scratch, void* stream) {
  if (state == nullptr || h == nullptr || router == nullptr || sel == nullptr || wts == nullptr || scratch == nullptr)
    return NH_E_ARG;
  if (n_expert <= 0 || n_expert > kMaxExperts || k <= 0 || k > kMaxTopK || k > n_expert || n_embd <= 0 ||
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
  const size_t smem = act_smem_bytes(p.K, true, true);
  const int grid = (n_expert + kRouterWarps - 1) / kRouterWarps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_router(p, smem, grid, st);
}

namespace {

template <int CPL>
int launch_gate_up(const GateUpArgs& p, size_t smem, int grid, cudaStream_t s) {
  static SmemLimit configured;
  if (!ensure_smem(gate_up_kernel<CPL>, smem, configured)) return NH_E_CUDA;
  return launch_pdl(gate_up_kernel<CPL>, dim3(grid), dim3(kMoeWarps * 32), smem, s, p);
}

template <int CPL>
int launch_down(const DownArgs& p, size_t smem, int grid, cudaStream_t s) {
  static SmemLimit configured;
  if (!ensure_smem(down_kernel<CPL>, smem, configured)) return NH_E_CUDA;
  return launch_pdl(down_kernel<CPL>, dim3(grid), dim3(kMoeWarps * 32), smem, s, p);
}

// Ring depth: as deep as kMoeMaxStages allows while the CTA stays near 100 KB
// of shared memory (so the next kernel's CTAs can be resident beside it), at
// least 2.
int pick_stages(size_t fixed, uint32_t stage_bytes) {
  int s = kMoeMaxStages;
  while (s > 2 && fixed + static_cast<size_t>(kMoeWarps) * s * (stage_bytes + 8) > 100 * 1024) --s;
  return s;
}

int grid_for(int jobs, size_t smem) {
  const int per_sm = static_cast<int>(std::min<size_t>(4, (220 * 1024) / (smem + 1024)));
  int grid = (jobs + kMoeWarps - 1) / kMoeWarps;
  const int cap = device_sm_count() * (per_sm < 1 ? 1 : per_sm);
  return grid > cap ? cap : (grid < 1 ? 1 : grid);
}

// Grid for a kernel at a dynamic shared-memory size: one warp per job, at
// most the CTAs that can be resident at once.
template <typename Kern>
int grid_resident(Kern k, int jobs, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kMoeWarps * 32, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  if (per_sm > ctas_per_sm_cap()) per_sm = ctas_per_sm_cap();
  int grid = (jobs + kMoeWarps - 1) / kMoeWarps;
  const int cap = device_sm_count() * per_sm;
  return grid > cap ? cap : (grid < 1 ? 1 : grid);
}

// Ring depth for the lane-per-super-block kernels: enough stages that the
// resident warps cover every job (two CTAs per SM), within ~110 KB.
int pick_stages3(size_t fixed, uint32_t stage_bytes, int jobs) {
  const int warps = device_sm_count() * ctas_per_sm_cap() * kMoeWarps;
  int s = (jobs + warps - 1) / warps;
  if (s < 1) s = 1;
  if (s > kMoeMaxStages) s = kMoeMaxStages;
  while (s > 1 && fixed + static_cast<size_t>(kMoeWarps) * s * (stage_bytes + 8) > 110 * 1024) --s;
  return s;
}

int launch_gate_up3(const GateUpArgs& p, size_t smem, cudaStream_t st) {
  static SmemLimit configured;
  if (!ensure_smem(gate_up3_kernel, smem, configured)) return NH_E_CUDA;
  const int grid = grid_resident(gate_up3_kernel, p.jobs_total, smem);
  return launch_pdl(gate_up3_kernel, dim3(grid), dim3(kMoeWarps * 32), smem, st, p);
}

int launch_down3(const DownArgs& p, size_t smem, cudaStream_t st) {
  static SmemLimit configured;
  if (!ensure_smem(down3_kernel, smem, configured)) return NH_E_CUDA;
  const int grid = grid_resident(down3_kernel, p.jobs_total, smem);
  return launch_pdl(down3_kernel, dim3(grid), dim3(kMoeWarps * 32), smem, st, p);
}

bool aligned16(const void* p, uint64_t stride) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (stride & 15) == 0;
}

// Lane-per-super-block gate/up jobs: G = K/256 lanes per row, P = 32/G gate
// rows and P up rows per job, staged gate then up (each 128-byte aligned).
void shape_gate_up3(GateUpArgs& p) {
  p.lpr = p.K / QK;
  p.rpp = 32 / p.lpr;
  p.R = p.rpp;
  const uint64_t gb = (p.rb_g * p.rpp + 32 + 127) & ~127ull;
  const uint64_t ub = (p.rb_u * p.rpp + 32 + 127) & ~127ull;
  p.up_off = static_cast<uint32_t>(gb);
  p.stage_bytes = static_cast<uint32_t>(gb + ub);
  p.jobs_per_expert = (p.F + p.rpp - 1) / p.rpp;
  p.jobs_total = p.jobs_per_expert * p.topk;
}

// The lane-per-super-block down kernel covers F/256 in {1,2,4,8} with the
// 32/G row groups of a pass divisible among the k experts.
bool down3_ok(int F, int k) { return rowdot3_k_ok(F) && (32 / (F / QK)) % k == 0; }

// Lane-per-super-block down jobs: G = F/256 lanes per row, 32/G row groups
// per pass shared by the k experts, so R = 32/(G*k) output rows per job.
void shape_down3(DownArgs& p) {
  p.lpr = p.F / QK;
  p.rpp = 32 / p.lpr;
  p.R = p.rpp / p.topk;
  // Expert slots are offset from 128-byte multiples so the lanes that read
  // the same super-block of different experts hit different banks: 64 mod
  // 128 for Q4_K (16-byte loads, two experts per quarter warp), 16 mod 128
  // for Q6_K (32-bit loads across the warp).
  p.slot_bytes = static_cast<uint32_t>(((p.rb * p.R + 32 + 127) & ~127ull) + (p.td == NH_TYPE_Q4_K ? 64 : 16));
  p.stage_bytes = p.slot_bytes * p.topk;
  p.jobs_total = (p.D + p.R - 1) / p.R;
  p.ystride = 0;
}

}  // namespace

// The selection comes from device memory (wsel) or, when slots_host is not
// null, from host memory, copied into the launch's arguments.
static int gate_up_entry(NhDecodeState* state, const float* h, const float* ffn_norm, float eps, const int32_t* wsel,
                         const int32_t* slots_host, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                         const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff, float* ff,
                         const void* down, uint64_t down_nb2, void* stream) {
  if (h == nullptr || (wsel == nullptr && slots_host == nullptr) || gate == nullptr || up == nullptr ||
      ff == nullptr)
    return NH_E_ARG;
  if (k <= 0 || k > kMaxTopK || n_embd <= 0 || n_embd > kMaxK || n_ff <= 0) return NH_E_ARG;
  const bool quant = tg != NH_TYPE_F32;
  if ((tg == NH_TYPE_F32) != (tu == NH_TYPE_F32)) return NH_E_TYPE;
  for (int t : {tg, tu})
    if (t != NH_TYPE_F32 && t != NH_TYPE_Q4_K && t != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (quant && !rowdot_k_ok(static_cast<int>(n_embd))) return NH_E_ARG;
  if ((tg == NH_TYPE_Q4_K && !aligned16(gate, gate_nb2)) || (tu == NH_TYPE_Q4_K && !aligned16(up, up_nb2)))
    return NH_E_ARG;
  GateUpArgs p;
  p.state = state;
  p.h = h;
  p.norm = ffn_norm;
  p.eps = eps;
  p.wsel = slots_host != nullptr ? nullptr : wsel;
  for (int i = 0; i < kMaxTopK; ++i) p.wsel_inline[i] = slots_host != nullptr && i < k ? slots_host[i] : 0;
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
  // Prefetch ranges start 16-byte aligned and have 16-byte multiple lengths.
  const bool pf = down != nullptr && down_nb2 > 0 && (reinterpret_cast<uintptr_t>(down) & 15) == 0 && (down_nb2 & 15) == 0;
  p.down = pf ? static_cast<const uint8_t*>(down) : nullptr;
  p.down_nb2 = pf ? down_nb2 : 0;
  if (quant && rowdot3_k_ok(p.K) && engine_v3()) {
    shape_gate_up3(p);
    p.ff = ff;
    const size_t fixed = ((act_smem_bytes(p.K, true, true) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double);
    p.S = pick_stages3(fixed, p.stage_bytes, p.jobs_total);
    const size_t smem = fixed + kMoeWarps * p.S * sizeof(uint64_t) + static_cast<size_t>(kMoeWarps) * p.S * p.stage_bytes;
    return launch_gate_up3(p, smem, static_cast<cudaStream_t>(stream));
  }
  if (quant) {
    p.lpr = rowdot_lpr(p.K);
    p.rpp = 32 / p.lpr;
    p.R = p.rpp >= 2 ? p.rpp / 2 : 1;
    if (p.R > 32) p.R = 32;
    const uint64_t gb = (p.rb_g * p.R + 32 + 127) & ~127ull;
    const uint64_t ub = (p.rb_u * p.R + 32 + 127) & ~127ull;
    p.up_off = static_cast<uint32_t>(gb);
    p.stage_bytes = static_cast<uint32_t>(gb + ub);
  } else {
    p.lpr = 32;
    p.rpp = 1;
    p.R = 1;
    p.up_off = 0;
    p.stage_bytes = 128;
  }
  p.jobs_per_expert = (p.F + p.R - 1) / p.R;
  p.jobs_total = p.jobs_per_expert * k;
  p.ff = ff;
  p.S = pick_stages(((act_smem_bytes(p.K, true, true) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double) +
                        kMoeWarps * 64 * sizeof(float),
                    p.stage_bytes);
  const size_t smem = ((act_smem_bytes(p.K, true, true) + 15) & ~static_cast<size_t>(15)) + 48 * sizeof(double) +
                      kMoeWarps * 64 * sizeof(float) + kMoeWarps * p.S * sizeof(uint64_t) +
                      static_cast<size_t>(kMoeWarps) * p.S * p.stage_bytes;
  const int grid = grid_for(p.jobs_total, smem);
  const int cpl = quant ? (p.K / 64 + 31) / 32 : 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return cpl <= 1 ? launch_gate_up<1>(p, smem, grid, s) : launch_gate_up<2>(p, smem, grid, s);
}

extern "C" int nh_moe_gate_up_prefetch(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                                       const int32_t* wsel, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                                       const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff,
                                       float* ff, const void* down, uint64_t down_nb2, void* stream) {
  if (wsel == nullptr) return NH_E_ARG;
  return gate_up_entry(state, h, ffn_norm, eps, wsel, nullptr, k, gate, tg, gate_nb2, up, tu, up_nb2, n_embd, n_ff,
                       ff, down, down_nb2, stream);
}

extern "C" int nh_moe_gate_up_slots(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                                    const int32_t* slots, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                                    const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff,
                                    float* ff, const void* down, uint64_t down_nb2, void* stream) {
  if (slots == nullptr) return NH_E_ARG;
  return gate_up_entry(state, h, ffn_norm, eps, nullptr, slots, k, gate, tg, gate_nb2, up, tu, up_nb2, n_embd, n_ff,
                       ff, down, down_nb2, stream);
}

extern "C" int nh_moe_gate_up(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                              const int32_t* wsel, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                              const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff, float* ff,
                              void* stream) {
  return nh_moe_gate_up_prefetch(state, h, ffn_norm, eps, wsel, k, gate, tg, gate_nb2, up, tu, up_nb2, n_embd, n_ff,
                                 ff, nullptr, 0, stream);
}

static int down_entry(const NhDecodeState* state, const float* ff, const int32_t* wsel, const int32_t* slots_host,
                      const float* wts, int k, const void* down, int32_t td, uint64_t down_nb2, int64_t n_ff,
                      int64_t n_embd, float* h_io, float* dump, int64_t dump_step_stride, int64_t dump_offset,
                      void* stream) {
  if (state == nullptr || ff == nullptr || (wsel == nullptr && slots_host == nullptr) || wts == nullptr ||
      down == nullptr || h_io == nullptr)
    return NH_E_ARG;
  if (k <= 0 || k > kMaxTopK || n_ff <= 0 || n_embd <= 0) return NH_E_ARG;
  if (td != NH_TYPE_F32 && td != NH_TYPE_Q4_K && td != NH_TYPE_Q6_K) return NH_E_TYPE;
  const bool quant = td != NH_TYPE_F32;
  if (quant && !rowdot_k_ok(static_cast<int>(n_ff))) return NH_E_ARG;
  if (static_cast<int64_t>(k) * n_ff > 4 * kMaxK) return NH_E_ARG;
  if (td == NH_TYPE_Q4_K && !aligned16(down, down_nb2)) return NH_E_ARG;
  DownArgs p;
  p.state = const_cast<NhDecodeState*>(state);
  p.ff = ff;
  p.wsel = slots_host != nullptr ? nullptr : wsel;
  for (int i = 0; i < kMaxTopK; ++i) p.wsel_inline[i] = slots_host != nullptr && i < k ? slots_host[i] : 0;
  p.wts = wts;
  p.topk = k;
  p.down = static_cast<const uint8_t*>(down);
  p.td = td;
  p.nb2 = down_nb2;
  p.rb = row_bytes(td, n_ff);
  p.F = static_cast<int>(n_ff);
  p.D = static_cast<int>(n_embd);
  if (quant && down3_ok(p.F, k) && engine_v3()) {
    shape_down3(p);
    p.h = h_io;
    p.dump = dump;
    p.dump_stride = dump_step_stride;
    p.dump_off = dump_offset;
    const size_t fixed = (act_smem_bytes(k * p.F, true) + 15) & ~static_cast<size_t>(15);
    p.S = pick_stages3(fixed, p.stage_bytes, p.jobs_total);
    const size_t smem = fixed + kMoeWarps * p.S * sizeof(uint64_t) + static_cast<size_t>(kMoeWarps) * p.S * p.stage_bytes;
    if (smem > 220 * 1024) return NH_E_ARG;
    return launch_down3(p, smem, static_cast<cudaStream_t>(stream));
  }
  if (quant) {
    p.lpr = rowdot_lpr(p.F);
    p.rpp = 32 / p.lpr;
    p.R = p.rpp >= k ? p.rpp / k : 1;
    if (p.R > 32) p.R = 32;
    p.slot_bytes = static_cast<uint32_t>((p.rb * p.R + 32 + 127) & ~127ull);
    p.stage_bytes = p.slot_bytes * k;
  } else {
    p.lpr = 32;
    p.rpp = 1;
    p.R = 1;
    p.slot_bytes = 128;
    p.stage_bytes = 128;
  }
  if (p.R * k > kMaxTopK * 32) return NH_E_ARG;
  p.jobs_total = (p.D + p.R - 1) / p.R;
  p.ystride = (k * p.R + 3) & ~3;
  p.S = pick_stages(((act_smem_bytes(k * p.F, !quant) + 15) & ~static_cast<size_t>(15)) +
                        static_cast<size_t>(kMoeWarps) * p.ystride * sizeof(float),
                    p.stage_bytes);
  p.h = h_io;
  p.dump = dump;
  p.dump_stride = dump_step_stride;
  p.dump_off = dump_offset;
  const int KF = k * p.F;
  const size_t smem = ((act_smem_bytes(KF, !quant) + 15) & ~static_cast<size_t>(15)) +
                      static_cast<size_t>(kMoeWarps) * kMaxTopK * 32 * sizeof(float) +
                      kMoeWarps * p.S * sizeof(uint64_t) +
                      static_cast<size_t>(kMoeWarps) * p.S * p.stage_bytes;
  if (smem > 220 * 1024) return NH_E_ARG;
  const int grid = grid_for(p.jobs_total, smem);
  const int cpl = quant ? (p.F / 64 + 31) / 32 : 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return cpl <= 1 ? launch_down<1>(p, smem, grid, s) : launch_down<2>(p, smem, grid, s);
}

extern "C" int nh_moe_down_combine(const NhDecodeState* state, const float* ff, const int32_t* wsel, const float* wts,
                                   int k, const void* down, int32_t td, uint64_t down_nb2, int64_t n_ff,
                                   int64_t n_embd, float* h_io, float* dump, int64_t dump_step_stride,
                                   int64_t dump_offset, void* stream) {
  if (wsel == nullptr) return NH_E_ARG;
  return down_entry(state, ff, wsel, nullptr, wts, k, down, td, down_nb2, n_ff, n_embd, h_io, dump, dump_step_stride,
                    dump_offset, stream);
}

extern "C" int nh_moe_down_combine_slots(const NhDecodeState* state, const float* ff, const int32_t* slots,
                                         const float* wts, int k, const void* down, int32_t td, uint64_t down_nb2,
                                         int64_t n_ff, int64_t n_embd, float* h_io, float* dump,
                                         int64_t dump_step_stride, int64_t dump_offset, void* stream) {
  if (slots == nullptr) return NH_E_ARG;
  return down_entry(state, ff, nullptr, slots, wts, k, down, td, down_nb2, n_ff, n_embd, h_io, dump,
                    dump_step_stride, dump_offset, stream);
}

// 16 counters, then the E tagged logits (8 bytes each).
extern "C" int64_t nh_moe_layer_scratch_bytes(int n_expert) { return 64 + 8 * static_cast<int64_t>(n_expert) + 64; }

namespace {

int launch_fused(FusedArgs& p, cudaStream_t st) {
  // Grid: enough warps for one job each (at least the router CTAs), at most
  // two CTAs per SM (the launch bounds); the rings take the remaining jobs.
  const int need = std::max((std::max(p.g.jobs_total, p.d.jobs_total) + kMoeWarps - 1) / kMoeWarps, p.router_ctas);
  int grid = std::min(need, 2 * device_sm_count());
  const size_t fixed = p.act_bytes + 48 * sizeof(double);
  // Ring depths for that grid, trimmed until two CTAs fit on an SM.
  const int warps = grid * kMoeWarps;
  p.g.S = std::min(kMoeMaxStages, std::max(1, (p.g.jobs_total + warps - 1) / warps));
  p.d.S = std::min(kMoeMaxStages, std::max(1, (p.d.jobs_total + warps - 1) / warps));
  // Each warp's region also holds one router row (n_embd floats).
  auto region = [&]() {
    const uint64_t r = std::max({static_cast<uint64_t>(p.g.S) * p.g.stage_bytes,
                                 static_cast<uint64_t>(p.d.S) * p.d.stage_bytes, static_cast<uint64_t>(p.r.K) * 4});
    return static_cast<uint32_t>((r + 127) & ~127ull);
  };
  auto total = [&]() {
    return fixed + kMoeWarps * (p.g.S + p.d.S + 1) * sizeof(uint64_t) + static_cast<size_t>(kMoeWarps) * region();
  };
  while ((p.g.S > 1 || p.d.S > 1) && total() > 112 * 1024) {
    if (static_cast<uint64_t>(p.g.S) * p.g.stage_bytes >= static_cast<uint64_t>(p.d.S) * p.d.stage_bytes && p.g.S > 1)
      --p.g.S;
    else if (p.d.S > 1)
      --p.d.S;
    else
      --p.g.S;
  }
  p.region_bytes = region();
  const size_t smem = total();
  if (smem > 220 * 1024) return NH_E_ARG;
  static SmemLimit configured;
  if (!ensure_smem(moe_fused_kernel, smem, configured)) return NH_E_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_fused_kernel, kMoeWarps * 32, smem) !=
          cudaSuccess ||
      per_sm < 1)
    return NH_E_ARG;
  grid = std::min(grid, per_sm * device_sm_count());
  if (grid < p.router_ctas) return NH_E_ARG;
  return launch_coop(moe_fused_kernel, dim3(grid), dim3(kMoeWarps * 32), smem, st, p);
}

}  // namespace

extern "C" int nh_moe_layer(const NhMoeLayer* L, void* stream) {
  if (L == nullptr || L->state == nullptr || L->h == nullptr || L->router == nullptr || L->gate == nullptr ||
      L->up == nullptr || L->down == nullptr || L->sel == nullptr || L->wts == nullptr || L->ff == nullptr ||
      L->scratch == nullptr)
    return NH_E_ARG;
  const int E = L->n_expert, k = L->k;
  if (E <= 0 || E > kMaxExperts || k <= 0 || k > kMaxTopK || k > E) return NH_E_ARG;
  if (L->n_embd <= 0 || L->n_embd > kMaxK || L->n_ff <= 0 || L->n_ff > kMaxK) return NH_E_ARG;
  for (int t : {L->tg, L->tu, L->td})
    if (t != NH_TYPE_Q4_K && t != NH_TYPE_Q6_K) return NH_E_TYPE;
  const int K = static_cast<int>(L->n_embd), F = static_cast<int>(L->n_ff);
  if (!engine_v3() || !rowdot3_k_ok(K) || !down3_ok(F, k) || static_cast<int64_t>(k) * F > 4 * kMaxK)
    return NH_E_ARG;
  // Router rows are staged by bulk copies: 16-byte aligned.
  if ((reinterpret_cast<uintptr_t>(L->router) & 15) != 0) return NH_E_ARG;
  if ((L->tg == NH_TYPE_Q4_K && !aligned16(L->gate, L->gate_nb2)) ||
      (L->tu == NH_TYPE_Q4_K && !aligned16(L->up, L->up_nb2)) ||
      (L->td == NH_TYPE_Q4_K && !aligned16(L->down, L->down_nb2)))
    return NH_E_ARG;
  FusedArgs p;
  RouterArgs& r = p.r;
  r.state = L->state;
  r.h = L->h;
  r.norm = L->ffn_norm;
  r.eps = L->eps;
  r.router = L->router;
  r.K = K;
  r.E = E;
  r.topk = k;
  r.norm_topk = L->norm_topk;
  r.layer = L->layer;
  r.n_layers = L->n_layers;
  r.sel = L->sel;
  r.wts = L->wts;
  r.trace_sel = L->trace_sel;
  r.trace_gap = L->trace_gap;
  r.ticket = static_cast<unsigned*>(L->scratch);
  r.logits = nullptr;  // published tagged (below), not through the standalone router's array
  p.tagged = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(L->scratch) + 64);
  p.epoch = static_cast<unsigned*>(L->scratch) + 15;
  p.sync = static_cast<unsigned*>(L->scratch) + 1;
  p.router_ctas = (E + kMoeWarps - 1) / kMoeWarps;
  GateUpArgs& g = p.g;
  g.state = L->state;
  g.h = L->h;
  g.norm = L->ffn_norm;
  g.eps = L->eps;
  g.wsel = L->sel;
  g.topk = k;
  g.gate = static_cast<const uint8_t*>(L->gate);
  g.up = static_cast<const uint8_t*>(L->up);
  g.tg = L->tg;
  g.tu = L->tu;
  g.gate_nb2 = L->gate_nb2;
  g.up_nb2 = L->up_nb2;
  g.K = K;
  g.F = F;
  g.rb_g = row_bytes(g.tg, K);
  g.rb_u = row_bytes(g.tu, K);
  g.ff = L->ff;
  g.down = nullptr;
  g.down_nb2 = 0;
  shape_gate_up3(g);
  DownArgs& d = p.d;
  d.state = L->state;
  d.ff = L->ff;
  d.wsel = L->sel;
  d.wts = L->wts;
  d.topk = k;
  d.down = static_cast<const uint8_t*>(L->down);
  d.td = L->td;
  d.nb2 = L->down_nb2;
  d.rb = row_bytes(d.td, F);
  d.F = F;
  d.D = K;
  d.h = L->h;
  d.dump = L->dump;
  d.dump_stride = L->dump_step_stride;
  d.dump_off = L->dump_offset;
  shape_down3(d);
  p.act_bytes = static_cast<uint32_t>(
      (std::max(act_smem_bytes(K, true, true), act_smem_bytes(k * F, false)) + 15) & ~static_cast<size_t>(15));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_fused(p, st);
}


NH_PHASE_TRACE_SETTER(moe)

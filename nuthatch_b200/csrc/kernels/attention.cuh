// Decode-step attention of one (query head, 64-position split) item, shared
// by the standalone attention kernel and the fused layer kernel: QK-norm over
// the full q/k width, NEOX RoPE, the KV append, scores, softmax and the V
// product, with the splits of a head combined in order by the last CTA to
// finish one (per-head tickets).  The arithmetic is written for
// kAttnThreads = 128 threads; a CTA with more threads runs it on its first
// 128 (the rest only take part in the CTA barriers).
#pragma once

#include "rowdot.cuh"

namespace nh {

constexpr int kAttnThreads = 128;
constexpr int kAttnSplit = 64;

// 64-position splits of a cache of max_seq positions.
inline int attn_splits(int max_seq) { return (max_seq + kAttnSplit - 1) / kAttnSplit; }

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

// Shared-memory layout of an item (floats): Ks [64][hd+4] (padded K rows:
// conflict-free 16-byte reads per position), Vs [64][hd], qh, kc, vc, qn, kn
// [hd], sc [64], qfull [n_head*hd], kfull [n_head_kv*hd].
struct AttnSmem {
  float *Ks, *Vs, *qh, *kc, *vc, *qn, *kn, *sc, *qfull, *kfull;
};

__host__ __device__ inline size_t attn_smem_floats(int hd, int n_head, int n_head_kv) {
  return static_cast<size_t>(kAttnSplit) * (hd + 4) + static_cast<size_t>(kAttnSplit) * hd + 5 * hd + kAttnSplit +
         static_cast<size_t>(n_head + n_head_kv) * hd;
}

__device__ inline AttnSmem carve_attn(float* sm, int hd, int n_head) {
  AttnSmem m;
  m.Ks = sm;
  m.Vs = m.Ks + kAttnSplit * (hd + 4);
  m.qh = m.Vs + kAttnSplit * hd;
  m.kc = m.qh + hd;
  m.vc = m.kc + hd;
  m.qn = m.vc + hd;
  m.kn = m.qn + hd;
  m.sc = m.kn + hd;
  m.qfull = m.sc + kAttnSplit;
  m.kfull = m.qfull + n_head * hd;
  return m;
}

struct AttnShared {
  uint64_t bar;
  double red[40];
  float s_max[4];
  int s_last;
};

// The part of an item that needs nothing from this step: the bulk copies of
// the cached K/V rows of the split (completing on sh.bar) and the norm
// weights.  Block-wide (contains a CTA barrier; attn_finish's first barrier
// orders the norm weights before their use).
__device__ inline void attn_begin(const AttnArgs& p, int h, int sp, int pos, const AttnSmem& m, AttnShared& sh) {
  const int tid = threadIdx.x;
  const int hd = p.hd;
  const int kst = hd + 4;
  const int group = p.n_head / p.n_head_kv;
  const int kh = h / group;
  const int dkv = p.n_head_kv * hd;
  const int n_kv = pos + 1;
  const int p0 = sp * kAttnSplit;
  const int p1 = min(n_kv, p0 + kAttnSplit);
  const int n_cached = max(0, min(p1, pos) - p0);
  const bool covers_cur = (p1 == n_kv);
  // Thread j < n_cached copies K row j, thread 64 + j V row j.
  const uint32_t row = static_cast<uint32_t>(hd) * 4;
  if (tid == 0) {
    mbar_init(&sh.bar, 1);
    fence_barrier_init();
    mbar_expect_tx(&sh.bar, 2u * row * static_cast<uint32_t>(n_cached));
  }
  __syncthreads();
  if (tid < 2 * kAttnSplit) {
    const int j = tid & (kAttnSplit - 1);
    if (j < n_cached) {
      const int64_t g = static_cast<int64_t>(p0 + j) * dkv + kh * hd;
      if (tid < kAttnSplit) bulk_g2s(m.Ks + j * kst, p.k_cache + g, row, &sh.bar);
      else bulk_g2s(m.Vs + j * hd, p.v_cache + g, row, &sh.bar);
    }
  }
  copy_to_smem(m.qn, p.q_norm + h * hd, hd);
  if (covers_cur) copy_to_smem(m.kn, p.k_norm + kh * hd, hd);
}

// The rest of an item, once q, k and v of this step are in memory.  Block-wide.
__device__ inline void attn_finish(const AttnArgs& p, int h, int sp, int pos, const AttnSmem& m, AttnShared& sh) {
  constexpr int nt = kAttnThreads, nw = kAttnThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool part = tid < nt;  // threads beyond nt only meet the barriers
  const int hd = p.hd;
  const int kst = hd + 4;
  const int group = p.n_head / p.n_head_kv;
  const int kh = h / group;
  const int dq = p.n_head * hd, dkv = p.n_head_kv * hd;
  const int half = hd / 2;
  const int n_kv = pos + 1;
  const int n_active = (n_kv + kAttnSplit - 1) / kAttnSplit;
  const int p0 = sp * kAttnSplit;
  const int p1 = min(n_kv, p0 + kAttnSplit);
  const int n = p1 - p0;
  const bool covers_cur = (p1 == n_kv);
  float* const Ks = m.Ks;
  float* const Vs = m.Vs;
  float* const qh = m.qh;
  float* const kc = m.kc;
  float* const vc = m.vc;
  float* const qn = m.qn;
  float* const kn = m.kn;
  float* const sc = m.sc;
  float* const qfull = m.qfull;
  float* const kfull = m.kfull;
  double* const red = sh.red;

  // q (and, for the CTA holding the current position, k and v) into shared
  // memory, every thread's loads of all three in flight before its first
  // store: one L2 latency instead of one per row.
  {
    const float* vsrc = p.v + kh * hd;
    const bool vec = ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
                       reinterpret_cast<uintptr_t>(vsrc)) & 15) == 0;
    if (vec) {
      const int nq4 = dq / 4, nk4 = covers_cur ? dkv / 4 : 0, nv4 = covers_cur ? hd / 4 : 0;
      const int tot = nq4 + nk4 + nv4, nthr = blockDim.x;
      auto src = [&](int i) -> const float4* {
        return i < nq4 ? reinterpret_cast<const float4*>(p.q) + i
               : i < nq4 + nk4 ? reinterpret_cast<const float4*>(p.k) + (i - nq4)
                               : reinterpret_cast<const float4*>(vsrc) + (i - nq4 - nk4);
      };
      auto dst = [&](int i) -> float4* {
        return i < nq4 ? reinterpret_cast<float4*>(qfull) + i
               : i < nq4 + nk4 ? reinterpret_cast<float4*>(kfull) + (i - nq4)
                               : reinterpret_cast<float4*>(vc) + (i - nq4 - nk4);
      };
      constexpr int U = 9;
      for (int base = tid; base < tot; base += U * nthr) {
        float4 buf[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * nthr;
          if (i < tot) buf[u] = __ldcg(src(i));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * nthr;
          if (i < tot) *dst(i) = buf[u];
        }
      }
    } else {
      copy_to_smem<true>(qfull, p.q, dq);
      if (covers_cur) {
        copy_to_smem<true>(kfull, p.k, dkv);
        copy_to_smem<true>(vc, vsrc, hd);
      }
    }
  }
  __syncthreads();
  phase_stamp(2);
  // RMS of the full q (and k) rows, sums of squares in double: per thread,
  // per warp, then the warp partials in order.
  if (part) {
    double sq = 0.0, sk = 0.0;
    for (int i = tid; i < dq; i += nt) sq += static_cast<double>(__fmul_rn(qfull[i], qfull[i]));
    if (covers_cur)
      for (int i = tid; i < dkv; i += nt) sk += static_cast<double>(__fmul_rn(kfull[i], kfull[i]));
    sq = warp_sum_d(sq);
    sk = warp_sum_d(sk);
    if (lane == 0) {
      red[warp] = sq;
      red[8 + warp] = sk;
    }
  }
  __syncthreads();
  const float* cs = p.rope_cs + static_cast<int64_t>(pos) * hd;
  if (part) {
    double tq = 0.0, tk = 0.0;
    for (int w = 0; w < nw; ++w) {
      tq += red[w];
      tk += red[8 + w];
    }
    const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(div_count(tq, dq)), p.eps)));
    // Normalise and rotate (NEOX pairs i, i + hd/2) in one step.
    for (int i = tid; i < half; i += nt) {
      const float c = cs[2 * i], s = cs[2 * i + 1];
      const float x0 = __fmul_rn(__fmul_rn(qfull[h * hd + i], scq), qn[i]);
      const float x1 = __fmul_rn(__fmul_rn(qfull[h * hd + i + half], scq), qn[i + half]);
      qh[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      qh[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    if (covers_cur) {
      const float sck =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(div_count(tk, dkv)), p.eps)));
      for (int i = tid; i < half; i += nt) {
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
        for (int i = tid; i < hd; i += nt) vd[i] = vc[i];
      }
    }
  }
  const bool ok = mbar_wait(&sh.bar, 0);
  if (!ok && tid == 0) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  __syncthreads();
  phase_stamp(3);

  // Scores kq = K.q * kq_scale.
  float my = -INFINITY;  // this thread's score (thread j: position p0 + j)
  if ((hd & 31) == 0) {
    if (tid < n) {
      const float* kr = (p0 + tid == pos) ? kc : Ks + tid * kst;
      const float d = score_thread(kr, qh, hd);
      my = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
    }
  } else {
    if (part) {
      for (int j = warp; j < n; j += nw) {
        const float* kr = (p0 + j == pos) ? kc : Ks + j * kst;
        float d = 0.f;
        for (int i = lane; i < hd; i += 32) d = __fadd_rn(d, __fmul_rn(kr[i], qh[i]));
        d = warp_sum(d);
        if (lane == 0) sc[j] = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
      }
    }
    __syncthreads();
    if (tid < n) my = sc[tid];
  }
  // n <= kAttnSplit (64) < nt: thread j holds position j.
  float mx = warp_max(my);
  if (part && lane == 0) sh.s_max[warp] = mx;
  __syncthreads();
  mx = sh.s_max[0];
  for (int w = 1; w < nw; ++w) mx = fmaxf(mx, sh.s_max[w]);
  const float e = tid < n ? exp_cw(__fsub_rn(my, mx)) : 0.f;
  double l = warp_sum_d(tid < n ? static_cast<double>(e) : 0.0);
  if (part && lane == 0) red[16 + warp] = l;
  __syncthreads();
  l = 0.0;
  for (int w = 0; w < nw; ++w) l += red[16 + w];
  if (tid < n) sc[tid] = n_active == 1 ? __fmul_rn(e, static_cast<float>(1.0 / l)) : e;
  __syncthreads();
  phase_stamp(4);

  float* out = p.out + h * hd;
  if (n_active == 1) {
    // ggml_soft_max scaled the exponentials by 1/sum before the V product (above).
    if (part) {
      for (int i = tid; i < hd; i += nt) {
        float acc = 0.f;
        for (int j = 0; j < n; ++j) {
          const float vv = (p0 + j == pos) ? vc[i] : Vs[j * hd + i];
          acc = __fadd_rn(acc, __fmul_rn(vv, sc[j]));
        }
        out[i] = acc;
      }
    }
    __syncthreads();
    return;
  }
  const int slot = h * p.n_split + sp;
  if (part) {
    for (int i = tid; i < hd; i += nt) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) {
        const float vv = (p0 + j == pos) ? vc[i] : Vs[j * hd + i];
        acc = __fadd_rn(acc, __fmul_rn(vv, sc[j]));
      }
      p.part_acc[static_cast<int64_t>(slot) * hd + i] = acc;
    }
  }
  if (tid == 0) {
    p.part_m[slot] = mx;
    p.part_l[slot] = l;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned t = atomicAdd(&p.tickets[h], 1u);
    sh.s_last = (t == static_cast<unsigned>(n_active - 1));
  }
  __syncthreads();
  if (!sh.s_last) return;
  __threadfence();
  // Combine the splits in order.  The staged K and V rows are no longer read:
  // they hold the weights and sums (up to 64*(hd+4) floats / 32*hd doubles).
  if (n_active <= kAttnSplit * (hd + 4) && n_active <= (kAttnSplit / 2) * hd) {
    const int64_t base = static_cast<int64_t>(h) * p.n_split;
    combine_splits(p.part_m + base, p.part_l + base, p.part_acc + base * hd, n_active, hd, Ks,
                   reinterpret_cast<double*>(Vs), out, tid, nt, part);
    if (tid == 0) p.tickets[h] = 0u;
    __syncthreads();
    return;
  }
  const volatile float* pm = p.part_m;
  const volatile double* pl = p.part_l;
  float M = -INFINITY;
  for (int s = 0; s < n_active; ++s) M = fmaxf(M, pm[h * p.n_split + s]);
  float* wsplit = sc;  // reuse: sized kAttnSplit, so combine in chunks
  double L = 0.0;
  for (int s0 = 0; s0 < n_active; s0 += kAttnSplit) {
    const int cnt = min(kAttnSplit, n_active - s0);
    __syncthreads();
    for (int s = tid; s < cnt; s += nt)
      if (part) wsplit[s] = exp_cw(__fsub_rn(pm[h * p.n_split + s0 + s], M));
    __syncthreads();
    for (int s = 0; s < cnt; ++s) L += pl[h * p.n_split + s0 + s] * static_cast<double>(wsplit[s]);
  }
  const float inv = static_cast<float>(1.0 / L);
  if (part) {
    for (int i = tid; i < hd; i += nt) {
      float acc = 0.f;
      for (int s0 = 0; s0 < n_active; s0 += kAttnSplit) {
        const int cnt = min(kAttnSplit, n_active - s0);
        for (int s = 0; s < cnt; ++s) {
          const float w = exp_cw(__fsub_rn(pm[h * p.n_split + s0 + s], M));
          acc = __fadd_rn(acc,
                          __fmul_rn(__ldcg(&p.part_acc[static_cast<int64_t>(h * p.n_split + s0 + s) * hd + i]), w));
        }
      }
      out[i] = __fmul_rn(acc, inv);
    }
  }
  if (tid == 0) p.tickets[h] = 0u;
  __syncthreads();
}

}  // namespace nh

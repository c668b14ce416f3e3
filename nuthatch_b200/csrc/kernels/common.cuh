// Shared device helpers for the sm_100a kernels: GGUF block formats, the Q8_K
// activation (the arithmetic ggml's CPU mul_mat applies to activations that
// meet a Q4_K/Q6_K weight), cp.async row staging and warp reductions.
//
// Rounding: every f32 product/sum that the reference rounds separately is
// written with __fmul_rn/__fadd_rn/__fsub_rn so nvcc cannot contract it into
// an FMA; integer sub-block sums are exact.
//
// Shared-memory layout of the Q8_K activation: block b's 256 quants are stored
// rotated by 16*(b mod 16) bytes (logical byte L of block b lives at
// b*256 + ((L + 16*(b & 15)) & 255)).  One lane owns one super-block of a
// weight row, so the lanes of a quarter-warp read the same logical offset of
// eight consecutive blocks; the rotation puts those reads in distinct banks.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../../include/nh_kernels.h"

namespace nh {

constexpr int QK = 256;
constexpr int kQ4KBytes = 144;
constexpr int kQ6KBytes = 210;
constexpr int kMaxK = 4096;  // longest activation row the kernels stage in shared memory

__host__ __device__ inline size_t row_bytes(int type, int64_t n) {
  return type == NH_TYPE_Q4_K   ? static_cast<size_t>(n / QK) * kQ4KBytes
         : type == NH_TYPE_Q6_K ? static_cast<size_t>(n / QK) * kQ6KBytes
                                : static_cast<size_t>(n) * 4;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFF)));
}

__device__ __forceinline__ int q8_rot(int b) { return (b & 15) * 16; }

// t / n, the mean of an RMSNorm's sum of squares.  For n a power of two,
// t * 2^-log2(n) and t / n are the same exact real number rounded once, so
// the multiplication gives the same double as the division.
__device__ __forceinline__ double div_count(double t, int n) {
  if (n > 0 && (n & (n - 1)) == 0) {
    const int e = __ffs(n) - 1;
    return t * __longlong_as_double(static_cast<long long>(1023 - e) << 52);
  }
  return t / static_cast<double>(n);
}
__device__ __forceinline__ int q8_off(int b, int L) { return b * QK + ((L + q8_rot(b)) & (QK - 1)); }

// exp_cw: exp(x) = 2^k * e^r with k = nearest(x / ln 2) and r = x - k*ln 2
// reduced in two steps (Cody & Waite, ln 2 = 355/512 - 2.1219444e-4), e^r
// from its degree-7 Taylor polynomial in Horner form; every step is an IEEE
// f32 operation, so the host restatement produces the same bits.
__device__ __forceinline__ float exp_cw(float x) {
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208404541015625f) return 0.f;
  const float kf = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(kf, 0.693359375f)), __fmul_rn(kf, -2.12194440e-4f));
  float p = 1.98412698e-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.38888889e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.33333333e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.16666667e-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.66666667e-1f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  return ldexpf(p, static_cast<int>(kf));
}

// ------------------------------------------------------------ warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------ cp.async staging
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Stages `bytes` bytes starting at `src` into `dst` (16-byte aligned shared
// buffer of at least bytes + 32).  The copy starts at src rounded down to 16
// bytes; the staged data begins at dst + (src & 15), which is returned.
// Callers guarantee the 16-byte-rounded range stays inside the allocation
// (device weight regions carry 256 bytes of tail padding).
__device__ __forceinline__ const uint8_t* stage_bytes_warp(uint8_t* dst, const uint8_t* src,
                                                           size_t bytes, int lane) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src);
  const uintptr_t al = a & ~static_cast<uintptr_t>(15);
  const int off = static_cast<int>(a - al);
  const int n16 = static_cast<int>((off + bytes + 15) >> 4);
  const uint8_t* g = reinterpret_cast<const uint8_t*>(al);
  for (int k = lane; k < n16; k += 32) cp_async16(dst + 16 * k, g + 16 * k);
  return dst + off;
}

// ------------------------------------------------------------ split combination
// The n_active split partials of one attention head (maximum m_s, double
// sum l_s, weighted V sums acc_s[hd], written by other CTAs and read through
// L2) combined in split order: M = max_s m_s, w_s = exp_cw(m_s - M),
// L = sum_s l_s * w_s (double, in order), out[i] = (sum_s acc_s[i] * w_s, in
// order) * (1/L).  The maxima/weights (ws, n_active floats) and the sums (ls,
// n_active doubles) are staged in shared memory first, all loads in flight at
// once.  Block-wide; threads with part = false only meet the barriers.
__device__ inline void combine_splits(const float* part_m, const double* part_l, const float* part_acc, int n_active,
                                      int hd, float* ws, double* ls, float* out, int tid, int nt, bool part) {
  for (int s = tid; s < n_active; s += nt) {
    if (!part) break;
    ws[s] = __ldcg(part_m + s);
    ls[s] = __ldcg(part_l + s);
  }
  __syncthreads();
  float M = -INFINITY;
  for (int s = 0; s < n_active; ++s) M = fmaxf(M, ws[s]);
  __syncthreads();
  for (int s = tid; s < n_active; s += nt) {
    if (!part) break;
    ws[s] = exp_cw(__fsub_rn(ws[s], M));
  }
  __syncthreads();
  double L = 0.0;
  for (int s = 0; s < n_active; ++s) L += ls[s] * static_cast<double>(ws[s]);
  const float inv = static_cast<float>(1.0 / L);
  if (part) {
    for (int i = tid; i < hd; i += nt) {
      float acc = 0.f;
      for (int s = 0; s < n_active; ++s)
        acc = __fadd_rn(acc, __fmul_rn(__ldcg(part_acc + static_cast<int64_t>(s) * hd + i), ws[s]));
      out[i] = __fmul_rn(acc, inv);
    }
  }
}

// ------------------------------------------------------------ activation (smem)
// One activation row in shared memory: its f32 values (the staged input, then
// the normalised row), the staged RMSNorm weight, and, for quantised weights,
// its Q8_K form (rotated int8 quants, per-256 scale, per-16 sums).
struct ActSmem {
  float* xf;       // [K] or nullptr
  float* wf;       // [K] or nullptr
  int8_t* qs;      // [K] rotated
  float* d;        // [K/256]
  int16_t* bsums;  // [K/16]
  int K;
};

__host__ __device__ inline size_t act_smem_bytes(int K, bool need_xf, bool need_wf = false) {
  return (need_xf ? static_cast<size_t>(K) * 4 + 16 : 0) + (need_wf ? static_cast<size_t>(K) * 4 + 16 : 0) + K +
         (K / QK + 1) * 4 + (K / 16 + 1) * 2 + 64;
}

__device__ inline ActSmem carve_act(uint8_t* base, int K, bool need_xf, bool need_wf = false) {
  ActSmem a;
  a.K = K;
  uintptr_t p = reinterpret_cast<uintptr_t>(base);
  a.xf = need_xf ? reinterpret_cast<float*>(p) : nullptr;
  if (need_xf) p = (p + static_cast<size_t>(K) * 4 + 15) & ~static_cast<uintptr_t>(15);
  a.wf = need_wf ? reinterpret_cast<float*>(p) : nullptr;
  if (need_wf) p = (p + static_cast<size_t>(K) * 4 + 15) & ~static_cast<uintptr_t>(15);
  a.qs = reinterpret_cast<int8_t*>(p);
  p += K;
  p = (p + 15) & ~static_cast<uintptr_t>(15);
  a.d = reinterpret_cast<float*>(p);
  p += (K / QK + 1) * 4;
  p = (p + 15) & ~static_cast<uintptr_t>(15);
  a.bsums = reinterpret_cast<int16_t*>(p);
  return a;
}

// Block-wide copy of n floats from global to shared memory.  Each thread
// issues all its (up to 8) 16-byte loads before its first store, so the row
// arrives in one memory latency instead of one per loop trip.  Falls back to
// scalar loads when src or dst is not 16-byte aligned or n is not a multiple
// of 4.  Does not synchronise.  CG: load through L2 only (ld.global.cg), for
// data another CTA of the same grid wrote after a grid-wide barrier.
template <bool CG = false>
__device__ inline void copy_to_smem(float* dst, const float* __restrict__ src, int n) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) != 0 || (n & 3) != 0) {
    for (int i = tid; i < n; i += nt) dst[i] = CG ? __ldcg(src + i) : src[i];
    return;
  }
  constexpr int U = 8;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  const int n4 = n >> 2;
  for (int base = tid; base < n4; base += U * nt) {
    float4 buf[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * nt;
      if (i < n4) buf[u] = CG ? __ldcg(s4 + i) : s4[i];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * nt;
      if (i < n4) d4[i] = buf[u];
    }
  }
}

// Block-wide RMS scale of the shared row x[0..K) with ggml_rms_norm semantics
// (sum of squares in double, mean rounded to f32, 1/sqrtf(mean + eps)).
// `red` holds >= 33 doubles.  Ends synchronised.
__device__ inline float block_rms_scale(const float* x, int K, float eps, double* red) {
  const int tid = threadIdx.x, nt = blockDim.x;
  double s = 0.0;
  for (int i = tid; i < K; i += nt) {
    const float v = x[i];
    s += static_cast<double>(__fmul_rn(v, v));
  }
  s = warp_sum_d(s);
  if ((tid & 31) == 0) red[tid >> 5] = s;
  __syncthreads();
  if (tid < 32) {
    double t = tid < (nt >> 5) ? red[tid] : 0.0;
    t = warp_sum_d(t);
    if (tid == 0) red[32] = t;
  }
  __syncthreads();
  const float mean = static_cast<float>(div_count(red[32], K));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// quantize_row_q8_K semantics for NB 256-value blocks held 8 per lane
// (v[i][k] = element lane*8 + k of block blk[i]): the first element of
// largest magnitude maps to -127 (iscale = -127/max, d = 1/iscale), round
// half to even, clamp at +127, 16 partial sums.  Writes the blocks with
// live[i] (warp-uniform) into the activation (rotated layout).  The NB
// blocks' steps are interleaved, so their shuffle and division latencies
// overlap; each block's arithmetic is the single-block one.
template <int NB>
__device__ __forceinline__ void quantize_blocks_warp(const float (&v)[NB][8], const int (&blk)[NB],
                                                     const bool (&live)[NB], ActSmem& a, int lane) {
  // Largest magnitude over each block, then the first element (lowest index:
  // lowest lane, then lowest k) that has it; mx is that element's value.
  float amax[NB], mx[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    amax[i] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax[i] = fmaxf(amax[i], fabsf(v[i][k]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int i = 0; i < NB; ++i) amax[i] = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], o));
  }
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    float cand = 0.f;
    bool has = false;
#pragma unroll
    for (int k = 7; k >= 0; --k) {
      if (fabsf(v[i][k]) == amax[i]) {
        cand = v[i][k];
        has = true;
      }
    }
    const unsigned who = __ballot_sync(0xffffffffu, has);
    mx[i] = __shfl_sync(0xffffffffu, cand, who != 0u ? __ffs(who) - 1 : 0);
  }
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    uint32_t w0 = 0, w1 = 0;
    int part = 0;
    float dq = 0.f;
    if (amax[i] != 0.f) {
      const float iscale = __fdiv_rn(-127.f, mx[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int q = min(127, __float2int_rn(__fmul_rn(iscale, v[i][k])));
        part += q;
        const uint32_t byte = static_cast<uint32_t>(q & 0xFF);
        if (k < 4) w0 |= byte << (8 * k);
        else w1 |= byte << (8 * (k - 4));
      }
      dq = __fdiv_rn(1.f, iscale);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    if (live[i]) {
      const int b = blk[i];
      *reinterpret_cast<uint2*>(a.qs + q8_off(b, lane * 8)) = make_uint2(w0, w1);
      if ((lane & 1) == 0) a.bsums[b * 16 + (lane >> 1)] = static_cast<int16_t>(part);
      if (lane == 0) a.d[b] = dq;
    }
  }
}

// One block (quantize_blocks_warp with NB = 1): block b, v[k] = element
// lane*8 + k.
__device__ __forceinline__ void quantize_block_warp(const float (&v)[8], int b, ActSmem& a, int lane) {
  const float (&vv)[1][8] = *reinterpret_cast<const float (*)[1][8]>(&v);
  const int blk[1] = {b};
  const bool live[1] = {true};
  quantize_blocks_warp<1>(vv, blk, live, a, lane);
}

// Stages the RMSNorm weight of an activation (static model data, so callers
// issue it before griddepcontrol.wait).  Does not synchronise; prep_act's
// first barrier orders it before use.
__device__ inline void act_load_norm(ActSmem& a, const float* __restrict__ norm_w) {
  if (a.wf != nullptr && norm_w != nullptr) copy_to_smem(a.wf, norm_w, a.K);
}

// Block-wide: the activation x = src (optionally RMS-normalised and, when
// has_norm_w, multiplied by the weight staged by act_load_norm: ggml_rms_norm
// + ggml_mul, y = (x*scale)*w), left as f32 in xf and Q8_K-quantised when
// `quant`.  Needs xf.  Ends synchronised.
// CG: src was written by another CTA of the same grid (see copy_to_smem).
template <bool CG = false>
__device__ inline void prep_act(ActSmem& a, const float* __restrict__ src, bool has_norm_w, bool do_norm,
                                float eps, bool quant, double* red) {
  const int K = a.K;
  const int tid = threadIdx.x, nt = blockDim.x, warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
  copy_to_smem<CG>(a.xf, src, K);
  __syncthreads();
  float scale = 1.f;
  if (do_norm) {
    // Sum of squares in double: per thread, per warp (butterfly), then the
    // warp partials in warp order by every thread.
    double s = 0.0;
    for (int i = tid; i < K; i += nt) {
      const float v = a.xf[i];
      s += static_cast<double>(__fmul_rn(v, v));
    }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += red[w];
    const float mean = static_cast<float>(div_count(t, K));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  const bool w = do_norm && has_norm_w && a.wf != nullptr;
  if (quant) {
    // Each warp normalises its own 256-value blocks and quantises them.
    for (int b = warp; b < K / QK; b += nw) {
      float* xb = a.xf + b * QK + lane * 8;
      const float4 v0 = *reinterpret_cast<const float4*>(xb);
      const float4 v1 = *reinterpret_cast<const float4*>(xb + 4);
      float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      if (do_norm) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          v[k] = __fmul_rn(v[k], scale);
          if (w) v[k] = __fmul_rn(v[k], a.wf[b * QK + lane * 8 + k]);
        }
        *reinterpret_cast<float4*>(xb) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(xb + 4) = make_float4(v[4], v[5], v[6], v[7]);
      }
      quantize_block_warp(v, b, a, lane);
    }
  } else if (do_norm) {
    for (int i = tid; i < K; i += nt) {
      float v = __fmul_rn(a.xf[i], scale);
      if (w) v = __fmul_rn(v, a.wf[i]);
      a.xf[i] = v;
    }
  }
  __syncthreads();
}

// Block-wide: Q8_K quantisation of the f32 row already in a.xf (left there by
// prep_act with quant = false), each warp its 256-value blocks: the same
// values and arithmetic as prep_act with quant = true.  Ends synchronised.
__device__ inline void quant_act_smem(ActSmem& a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int b = warp; b < a.K / QK; b += nw) {
    const float* xb = a.xf + b * QK + lane * 8;
    const float4 v0 = *reinterpret_cast<const float4*>(xb);
    const float4 v1 = *reinterpret_cast<const float4*>(xb + 4);
    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    quantize_block_warp(v, b, a, lane);
  }
  __syncthreads();
}

// ------------------------------------------------------------ super-block dots
// One lane computes one whole super-block's contribution.  `blk` points into
// shared memory; `q8` is the base of the activation's quants, `b` the
// activation block index (for the rotation), `bs` its 16-sums, `yd` its
// scale.  Result as the oracle forms it per super-block:
// (d*yd)*sumi - (dmin*yd)*summ.
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[4 + j] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

__device__ __forceinline__ int4 ld_q8_16(const int8_t* q8, int b, int L) {
  return *reinterpret_cast<const int4*>(q8 + q8_off(b, L));
}

__device__ __forceinline__ float sb_dot_q4k(const uint8_t* blk, const int8_t* q8, int b, const int16_t* bs,
                                            float yd) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  const float d = half_bits_to_float(hdr.x);
  const float dmin = half_bits_to_float(hdr.x >> 16);
  uint8_t s[12];
  *reinterpret_cast<uint32_t*>(s + 0) = hdr.y;
  *reinterpret_cast<uint32_t*>(s + 4) = hdr.z;
  *reinterpret_cast<uint32_t*>(s + 8) = hdr.w;
  int sumi = 0, summ = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
    const uint4 w1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
    const int4 xa = ld_q8_16(q8, b, 64 * c);
    const int4 xb = ld_q8_16(q8, b, 64 * c + 16);
    const int4 xc = ld_q8_16(q8, b, 64 * c + 32);
    const int4 xd = ld_q8_16(q8, b, 64 * c + 48);
    const uint32_t m4 = 0x0F0F0F0Fu;
    int lo = 0, hi = 0;
    lo = __dp4a(static_cast<int>(w0.x & m4), xa.x, lo);
    lo = __dp4a(static_cast<int>(w0.y & m4), xa.y, lo);
    lo = __dp4a(static_cast<int>(w0.z & m4), xa.z, lo);
    lo = __dp4a(static_cast<int>(w0.w & m4), xa.w, lo);
    lo = __dp4a(static_cast<int>(w1.x & m4), xb.x, lo);
    lo = __dp4a(static_cast<int>(w1.y & m4), xb.y, lo);
    lo = __dp4a(static_cast<int>(w1.z & m4), xb.z, lo);
    lo = __dp4a(static_cast<int>(w1.w & m4), xb.w, lo);
    hi = __dp4a(static_cast<int>((w0.x >> 4) & m4), xc.x, hi);
    hi = __dp4a(static_cast<int>((w0.y >> 4) & m4), xc.y, hi);
    hi = __dp4a(static_cast<int>((w0.z >> 4) & m4), xc.z, hi);
    hi = __dp4a(static_cast<int>((w0.w >> 4) & m4), xc.w, hi);
    hi = __dp4a(static_cast<int>((w1.x >> 4) & m4), xd.x, hi);
    hi = __dp4a(static_cast<int>((w1.y >> 4) & m4), xd.y, hi);
    hi = __dp4a(static_cast<int>((w1.z >> 4) & m4), xd.z, hi);
    hi = __dp4a(static_cast<int>((w1.w >> 4) & m4), xd.w, hi);
    int sc0, m0, sc1, m1;
    q4k_scale_min(s, 2 * c, sc0, m0);
    q4k_scale_min(s, 2 * c + 1, sc1, m1);
    sumi += sc0 * lo + sc1 * hi;
    summ += m0 * (bs[4 * c] + bs[4 * c + 1]) + m1 * (bs[4 * c + 2] + bs[4 * c + 3]);
  }
  const float dd = __fmul_rn(d, yd), dm = __fmul_rn(dmin, yd);
  return __fsub_rn(__fmul_rn(dd, static_cast<float>(sumi)), __fmul_rn(dm, static_cast<float>(summ)));
}

// Unaligned 32-bit read from shared memory (the address is at least 2-byte aligned).
__device__ __forceinline__ uint32_t ld32u(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  return __funnelshift_r(w[0], w[1], static_cast<uint32_t>((a & 3) * 8));
}

__device__ __forceinline__ float sb_dot_q6k(const uint8_t* blk, const int8_t* q8, int b, const int16_t* bs,
                                            float yd) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  int grp[16];
#pragma unroll
  for (int g = 0; g < 16; ++g) grp[g] = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int l4 = 0; l4 < 8; ++l4) {
      const uint32_t A = ld32u(ql + 64 * h + 4 * l4);
      const uint32_t B = ld32u(ql + 64 * h + 32 + 4 * l4);
      const uint32_t H = ld32u(qh + 32 * h + 4 * l4);
      const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
      const uint32_t q0 = (A & m4) | ((H << 4) & m2);
      const uint32_t q1 = (B & m4) | ((H << 2) & m2);
      const uint32_t q2 = ((A >> 4) & m4) | (H & m2);
      const uint32_t q3 = ((B >> 4) & m4) | ((H >> 2) & m2);
      const int base = 128 * h + 4 * l4;
      const int g = 8 * h + (l4 >> 2);
      grp[g + 0] = __dp4a(static_cast<int>(q0), *reinterpret_cast<const int*>(q8 + q8_off(b, base)), grp[g + 0]);
      grp[g + 2] = __dp4a(static_cast<int>(q1), *reinterpret_cast<const int*>(q8 + q8_off(b, base + 32)), grp[g + 2]);
      grp[g + 4] = __dp4a(static_cast<int>(q2), *reinterpret_cast<const int*>(q8 + q8_off(b, base + 64)), grp[g + 4]);
      grp[g + 6] = __dp4a(static_cast<int>(q3), *reinterpret_cast<const int*>(q8 + q8_off(b, base + 96)), grp[g + 6]);
    }
  }
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
  int sumi = 0;
#pragma unroll
  for (int g = 0; g < 16; ++g) sumi += static_cast<int>(sc[g]) * (grp[g] - 32 * bs[g]);
  const uint32_t dbits = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(blk + 208));
  return __fmul_rn(__fmul_rn(half_bits_to_float(dbits), yd), static_cast<float>(sumi));
}

// Lanes per row for a row of `nsb` super-blocks: the next power of two, capped at 32.
__host__ __device__ inline int lanes_per_row(int nsb) {
  int l = 1;
  while (l < nsb && l < 32) l <<= 1;
  return l;
}

// Dot of one staged quantised row with the activation blocks b0 .. b0+nsb-1:
// lane `sub` of `lpr` lanes handles super-blocks sub, sub+lpr, ...; result
// reduced over the lpr lanes (valid in every one of them).
__device__ __forceinline__ float row_dot_q(const uint8_t* row, int type, int nsb, int sub, int lpr,
                                           const ActSmem& a, int b0) {
  float acc = 0.f;
  for (int s = sub; s < nsb; s += lpr) {
    const int b = b0 + s;
    const float v = type == NH_TYPE_Q4_K ? sb_dot_q4k(row + s * kQ4KBytes, a.qs, b, a.bsums + b * 16, a.d[b])
                                         : sb_dot_q6k(row + s * kQ6KBytes, a.qs, b, a.bsums + b * 16, a.d[b]);
    acc = __fadd_rn(acc, v);
  }
  for (int o = 1; o < lpr; o <<= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  return acc;
}

// f32 row (global memory) dot the f32 activation; whole warp, result in every lane.
__device__ __forceinline__ float row_dot_f32(const float* __restrict__ w, const float* x, int K, int lane) {
  float s = 0.f;
  for (int i = lane; i < K; i += 32) s = __fadd_rn(s, __fmul_rn(w[i], x[i]));
  return warp_sum(s);
}

// Block-wide argmax of (value, index) pairs with the first-maximum rule
// (greater value wins, equal values keep the lower index); result valid in
// thread 0.  `sv`/`si` hold >= 32 entries.
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}
__device__ inline void block_argmax(float& v, int& i, float* sv, int* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (argmax_better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w)
      if (argmax_better(sv[w], si[w], v, i)) {
        v = sv[w];
        i = si[w];
      }
  }
}

}  // namespace nh

// Row-dot engine of the GEMV kernels.
//
// Work mapping: a quantised row of K values is split into 64-value chunks (a
// Q4_K super-block holds 4).  Lane l of a warp owns chunk position j = l %
// LPR of a row (LPR = min(32, K/64) lanes per row; 32/LPR rows per pass), so
// the lane's slice of the Q8_K activation is the same for every row and stays
// in registers for the whole kernel.  The integer dot of each chunk is exact;
// the four chunks of a super-block are summed as integers with shuffles, the
// super-block is scaled in f32 exactly as the oracle does, and super-blocks
// are summed with shuffles.
//
// Weight staging: each warp runs its own ring of kStages shared buffers, one
// job (a group of rows, or one row of several experts) per buffer, filled by
// cp.async.bulk (TMA, 1-D) copies that complete on a per-buffer mbarrier.  The
// copies start 16-byte aligned below the first row and end 16-byte aligned
// above the last, so device weight regions carry >= 32 bytes of tail padding.
// Every mbarrier wait is bounded: on expiry the kernel records NH_E_TIMEOUT
// in its error word and stops working.
#pragma once

#include "common.cuh"

namespace nh {

constexpr int kWaitSpins = 1 << 22;

// ------------------------------------------------------------------ PDL
// Programmatic dependent launch: wait for the preceding kernel's results, and
// let the following kernel start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// ------------------------------------------------------------------ mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kWaitSpins; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// L2 prefetch of a global range (no shared memory involved).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}

// One 16-byte aligned span covering [src, src+bytes): returns the aligned
// start and sets *len to its 16-byte multiple length and *off to the offset of
// src inside it.
__device__ __forceinline__ const uint8_t* span16(const uint8_t* src, size_t bytes, uint32_t* len, uint32_t* off) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src);
  const uintptr_t al = a & ~static_cast<uintptr_t>(15);
  *off = static_cast<uint32_t>(a - al);
  *len = static_cast<uint32_t>((a + bytes - al + 15) & ~static_cast<uintptr_t>(15));
  return reinterpret_cast<const uint8_t*>(al);
}

// ------------------------------------------------------------------ register activation
// The lane's activation: CPL chunks of 64 Q8_K quants (16 words each), their
// 16-sums, and the scale of each chunk's super-block.
template <int CPL>
struct ActReg {
  int x[CPL][16];
  int bs[CPL][4];
  float yd[CPL];
};

// Loads chunks c_glob = b0*4 + j + LPR*t (t < CPL) of the shared activation.
template <int CPL>
__device__ __forceinline__ void load_act(ActReg<CPL>& r, const ActSmem& a, int b0, int j, int lpr) {
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int cg = j + lpr * t;
    const int b = b0 + cg / 4, L = 64 * (cg % 4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int4 v = *reinterpret_cast<const int4*>(a.qs + q8_off(b, L + 16 * q));
      r.x[t][4 * q + 0] = v.x;
      r.x[t][4 * q + 1] = v.y;
      r.x[t][4 * q + 2] = v.z;
      r.x[t][4 * q + 3] = v.w;
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) r.bs[t][g] = a.bsums[b * 16 + (L / 16) + g];
    r.yd[t] = a.d[b];
  }
}

// Integer parts of one Q4_K chunk c (0..3) of the super-block at blk (16-byte
// aligned shared memory): sumi = sc*<q,x> over its two sub-blocks, summ =
// m*bsum.
__device__ __forceinline__ void chunk_q4k(const uint8_t* blk, int c, const int (&x)[16], const int (&bs)[4],
                                          int& sumi, int& summ, float& d, float& dmin) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  d = half_bits_to_float(hdr.x);
  dmin = half_bits_to_float(hdr.x >> 16);
  uint8_t s[12];
  *reinterpret_cast<uint32_t*>(s + 0) = hdr.y;
  *reinterpret_cast<uint32_t*>(s + 4) = hdr.z;
  *reinterpret_cast<uint32_t*>(s + 8) = hdr.w;
  const uint4 w0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
  const uint4 w1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
  const uint32_t m4 = 0x0F0F0F0Fu;
  int lo = 0, hi = 0;
  lo = __dp4a(static_cast<int>(w0.x & m4), x[0], lo);
  lo = __dp4a(static_cast<int>(w0.y & m4), x[1], lo);
  lo = __dp4a(static_cast<int>(w0.z & m4), x[2], lo);
  lo = __dp4a(static_cast<int>(w0.w & m4), x[3], lo);
  lo = __dp4a(static_cast<int>(w1.x & m4), x[4], lo);
  lo = __dp4a(static_cast<int>(w1.y & m4), x[5], lo);
  lo = __dp4a(static_cast<int>(w1.z & m4), x[6], lo);
  lo = __dp4a(static_cast<int>(w1.w & m4), x[7], lo);
  hi = __dp4a(static_cast<int>((w0.x >> 4) & m4), x[8], hi);
  hi = __dp4a(static_cast<int>((w0.y >> 4) & m4), x[9], hi);
  hi = __dp4a(static_cast<int>((w0.z >> 4) & m4), x[10], hi);
  hi = __dp4a(static_cast<int>((w0.w >> 4) & m4), x[11], hi);
  hi = __dp4a(static_cast<int>((w1.x >> 4) & m4), x[12], hi);
  hi = __dp4a(static_cast<int>((w1.y >> 4) & m4), x[13], hi);
  hi = __dp4a(static_cast<int>((w1.z >> 4) & m4), x[14], hi);
  hi = __dp4a(static_cast<int>((w1.w >> 4) & m4), x[15], hi);
  int sc0, m0, sc1, m1;
  q4k_scale_min(s, 2 * c, sc0, m0);
  q4k_scale_min(s, 2 * c + 1, sc1, m1);
  sumi = sc0 * lo + sc1 * hi;
  summ = m0 * (bs[0] + bs[1]) + m1 * (bs[2] + bs[3]);
}

// Words of an at-least-2-byte-aligned shared-memory range.
template <int N>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&w)[N]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~static_cast<uintptr_t>(3));
  if ((a & 3) == 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = base[i];
  } else {
    uint32_t prev = base[0];
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const uint32_t next = base[i + 1];
      w[i] = __byte_perm(prev, next, 0x5432);
      prev = next;
    }
  }
}

// Integer part of one Q6_K chunk c (0..3) of the super-block at blk (2-byte
// aligned): sumi = sum_g sc_g * (<q6,x>_g - 32*bsum_g) over its four 16-groups.
__device__ __forceinline__ void chunk_q6k(const uint8_t* blk, int c, const int (&x)[16], const int (&bs)[4],
                                          int& sumi, float& d) {
  const int h = c >> 1, p = c & 1;
  uint32_t A[16], H[8];
  load_words<16>(blk + 64 * h, A);
  load_words<8>(blk + 128 + 32 * h, H);
  const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
  int g[4] = {0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t qa, qb;  // sub-chunks 2p (e = 64p + l) and 2p+1 (e = 64p + 32 + l), l = 4k..4k+3
    if (p == 0) {
      qa = (A[k] & m4) | ((H[k] << 4) & m2);
      qb = (A[8 + k] & m4) | ((H[k] << 2) & m2);
    } else {
      qa = ((A[k] >> 4) & m4) | (H[k] & m2);
      qb = ((A[8 + k] >> 4) & m4) | ((H[k] >> 2) & m2);
    }
    g[k >> 2] = __dp4a(static_cast<int>(qa), x[k], g[k >> 2]);
    g[2 + (k >> 2)] = __dp4a(static_cast<int>(qb), x[8 + k], g[2 + (k >> 2)]);
  }
  const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 4 * c);
  sumi = static_cast<int>(sc[0]) * (g[0] - 32 * bs[0]) + static_cast<int>(sc[1]) * (g[1] - 32 * bs[1]) +
         static_cast<int>(sc[2]) * (g[2] - 32 * bs[2]) + static_cast<int>(sc[3]) * (g[3] - 32 * bs[3]);
  d = half_bits_to_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(blk + 208)));
}

// Dot of one staged quantised row (`row` in shared memory) with the lane's
// register activation.  Lanes j = lane % LPR of the row's lane group each take
// chunks j + LPR*t.  Result valid in every lane of the group.
template <int CPL>
__device__ __forceinline__ float row_dot_reg(const uint8_t* row, int type, int j, int lpr, const ActReg<CPL>& ar) {
  float acc = 0.f;
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int cg = j + lpr * t;
    const int s = cg >> 2, c = cg & 3;
    int sumi, summ = 0;
    float d, dmin = 0.f;
    if (type == NH_TYPE_Q4_K) {
      chunk_q4k(row + s * kQ4KBytes, c, ar.x[t], ar.bs[t], sumi, summ, d, dmin);
    } else {
      chunk_q6k(row + s * kQ6KBytes, c, ar.x[t], ar.bs[t], sumi, d);
    }
    // The four chunks of a super-block sit in four consecutive lanes.
    sumi += __shfl_xor_sync(0xffffffffu, sumi, 1);
    sumi += __shfl_xor_sync(0xffffffffu, sumi, 2);
    summ += __shfl_xor_sync(0xffffffffu, summ, 1);
    summ += __shfl_xor_sync(0xffffffffu, summ, 2);
    const float yd = ar.yd[t];
    float v = type == NH_TYPE_Q4_K
                  ? __fsub_rn(__fmul_rn(__fmul_rn(d, yd), static_cast<float>(sumi)),
                              __fmul_rn(__fmul_rn(dmin, yd), static_cast<float>(summ)))
                  : __fmul_rn(__fmul_rn(d, yd), static_cast<float>(sumi));
    if ((j & 3) != 0) v = 0.f;
    acc = __fadd_rn(acc, v);
  }
  for (int o = 4; o < lpr; o <<= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  return acc;
}

// Supported quantised row lengths: K/64 chunks a power of two, K <= kMaxK.
__host__ __device__ inline bool rowdot_k_ok(int K) {
  if (K < QK || K > kMaxK || K % QK != 0) return false;
  const int c = K / 64;
  return (c & (c - 1)) == 0;
}
__host__ __device__ inline int rowdot_lpr(int K) { return K / 64 < 32 ? K / 64 : 32; }

}  // namespace nh

// Row-dot engine, lane-per-super-block form.
//
// Work mapping: a quantised row of K <= 2048 values has NSB = K/256
// super-blocks.  G = NSB lanes work on one row, lane g owning super-block g,
// so a warp pass covers 32/G rows at once (4 rows for K = 2048, 8 for 1024).
// Each lane holds its super-block of the Q8_K activation in registers (64
// words of quants, the 16 partial sums, the scale) for the whole kernel,
// computes the super-block's exact integer dot and scales it in f32 exactly
// as the oracle does, and the G lanes of a row are combined by a butterfly
// over lane strides 1, 2, 4: the pairwise super-block tree of the oracle's
// RowSum, so results are identical to it bit for bit.
//
// Q4_K super-blocks (144 bytes) start 16-byte aligned when the weight base
// is 16-byte aligned and are read with 16-byte shared loads.  Q6_K
// super-blocks (210 bytes) start 2-byte aligned; their words are assembled
// with funnel shifts from aligned 32-bit loads (reading at most 4 bytes past
// the super-block, inside the staging buffer's padding).
#pragma once

#include "rowdot.cuh"

namespace nh {

constexpr int kMaxG = 8;  // lanes per row = super-blocks per row (K <= 2048)

struct Act3 {
  int x[64];     // 256 int8 quants, 4 per word
  int bs[8];     // 16 int16 partial sums, 2 per word (low half = even group)
  float yd;      // the super-block's scale
};

// Loads super-block b of the shared Q8_K activation (rotated layout).
__device__ __forceinline__ void load_act3(Act3& r, const ActSmem& a, int b) {
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int4 v = *reinterpret_cast<const int4*>(a.qs + q8_off(b, 16 * q));
    r.x[4 * q + 0] = v.x;
    r.x[4 * q + 1] = v.y;
    r.x[4 * q + 2] = v.z;
    r.x[4 * q + 3] = v.w;
  }
  const int4 s0 = *reinterpret_cast<const int4*>(a.bsums + b * 16);
  const int4 s1 = *reinterpret_cast<const int4*>(a.bsums + b * 16 + 8);
  r.bs[0] = s0.x;
  r.bs[1] = s0.y;
  r.bs[2] = s0.z;
  r.bs[3] = s0.w;
  r.bs[4] = s1.x;
  r.bs[5] = s1.y;
  r.bs[6] = s1.z;
  r.bs[7] = s1.w;
  r.yd = a.d[b];
}

// The super-block dots read the activation through one of two views with the
// same values: the lane's registers (Act3, for warps that reuse it over many
// rows) or shared memory directly (for warps that dot only a row or two,
// where holding 73 registers would only crowd the rest of the kernel).
struct Act3Regs {
  const Act3& r;
  __device__ __forceinline__ int4 x4(int q) const {
    return make_int4(r.x[4 * q], r.x[4 * q + 1], r.x[4 * q + 2], r.x[4 * q + 3]);
  }
  __device__ __forceinline__ int bs(int j) const { return r.bs[j]; }
  __device__ __forceinline__ float yd() const { return r.yd; }
};

struct Act3Smem {
  const ActSmem& a;
  int b;  // the activation super-block
  __device__ __forceinline__ int4 x4(int q) const { return *reinterpret_cast<const int4*>(a.qs + q8_off(b, 16 * q)); }
  __device__ __forceinline__ int bs(int j) const { return *reinterpret_cast<const int*>(a.bsums + b * 16 + 2 * j); }
  __device__ __forceinline__ float yd() const { return a.d[b]; }
};

__device__ __forceinline__ int lo16(int w) { return static_cast<int>(static_cast<int16_t>(w & 0xFFFF)); }
__device__ __forceinline__ int hi16(int w) { return w >> 16; }
__device__ __forceinline__ int byte_of(uint32_t w, int i) { return static_cast<int>((w >> (8 * i)) & 0xFF); }

// One Q4_K super-block (16-byte aligned shared memory) against the lane's
// activation: (d*yd)*sumi - (dmin*yd)*summ with
// sumi = sum_j sc_j * <q4, q8>_j and summ = sum_j m_j * bsum_j.
template <class View>
__device__ __forceinline__ float sb_dot_q4k3(const uint8_t* blk, const View& a) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  // 6-bit scales and mins of sub-blocks 0-3 (sc0, m0) and 4-7 (sc1, m1), one per byte.
  const uint32_t sc0 = hdr.y & 0x3F3F3F3Fu;
  const uint32_t m0 = hdr.z & 0x3F3F3F3Fu;
  const uint32_t sc1 = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
  const uint32_t m1 = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  const uint32_t m4 = 0x0F0F0F0Fu;
  int sumi = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
    const uint4 w1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
    const int4 x0 = a.x4(4 * c), x1 = a.x4(4 * c + 1), x2 = a.x4(4 * c + 2), x3 = a.x4(4 * c + 3);
    int lo = 0, hi = 0;
    lo = __dp4a(static_cast<int>(w0.x & m4), x0.x, lo);
    lo = __dp4a(static_cast<int>(w0.y & m4), x0.y, lo);
    lo = __dp4a(static_cast<int>(w0.z & m4), x0.z, lo);
    lo = __dp4a(static_cast<int>(w0.w & m4), x0.w, lo);
    lo = __dp4a(static_cast<int>(w1.x & m4), x1.x, lo);
    lo = __dp4a(static_cast<int>(w1.y & m4), x1.y, lo);
    lo = __dp4a(static_cast<int>(w1.z & m4), x1.z, lo);
    lo = __dp4a(static_cast<int>(w1.w & m4), x1.w, lo);
    hi = __dp4a(static_cast<int>((w0.x >> 4) & m4), x2.x, hi);
    hi = __dp4a(static_cast<int>((w0.y >> 4) & m4), x2.y, hi);
    hi = __dp4a(static_cast<int>((w0.z >> 4) & m4), x2.z, hi);
    hi = __dp4a(static_cast<int>((w0.w >> 4) & m4), x2.w, hi);
    hi = __dp4a(static_cast<int>((w1.x >> 4) & m4), x3.x, hi);
    hi = __dp4a(static_cast<int>((w1.y >> 4) & m4), x3.y, hi);
    hi = __dp4a(static_cast<int>((w1.z >> 4) & m4), x3.z, hi);
    hi = __dp4a(static_cast<int>((w1.w >> 4) & m4), x3.w, hi);
    const uint32_t scw = c < 2 ? sc0 : sc1;
    sumi += byte_of(scw, (2 * c) & 3) * lo + byte_of(scw, (2 * c + 1) & 3) * hi;
  }
  int summ = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int m = byte_of(j < 4 ? m0 : m1, j & 3);
    const int bw = a.bs(j);
    summ += m * (lo16(bw) + hi16(bw));
  }
  const float d = half_bits_to_float(hdr.x);
  const float dmin = half_bits_to_float(hdr.x >> 16);
  const float yd = a.yd();
  return __fsub_rn(__fmul_rn(__fmul_rn(d, yd), static_cast<float>(sumi)),
                   __fmul_rn(__fmul_rn(dmin, yd), static_cast<float>(summ)));
}

// One Q6_K super-block (2-byte aligned shared memory):
// (d*yd) * sum_g sc_g * (<q6, q8>_g - 32*bsum_g) over its sixteen 16-groups.
template <class View>
__device__ __forceinline__ float sb_dot_q6k3(const uint8_t* blk, const View& a) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;
  auto word = [&](int i) { return __funnelshift_r(base[i], base[i + 1], sh); };
  const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
  const uint32_t scw[4] = {word(48), word(49), word(50), word(51)};  // int8 scales, group g in byte g%4 of word g/4
  int sumi = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // k = 4*half .. 4*half+3: groups 8h + half + {0, 2, 4, 6}
      int g1 = 0, g2 = 0, g3 = 0, g4 = 0;
      // Activation words 32h + {0, 8, 16, 24} + 4*half + kk.
      const int4 xa = a.x4(8 * h + half), xb = a.x4(8 * h + 2 + half);
      const int4 xc = a.x4(8 * h + 4 + half), xd = a.x4(8 * h + 6 + half);
      const int xs[4][4] = {{xa.x, xa.y, xa.z, xa.w}, {xb.x, xb.y, xb.z, xb.w},
                            {xc.x, xc.y, xc.z, xc.w}, {xd.x, xd.y, xd.z, xd.w}};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int k = 4 * half + kk;
        const uint32_t A = word(16 * h + k);      // ql bytes 64h + 4k ..
        const uint32_t B = word(16 * h + 8 + k);  // ql bytes 64h + 32 + 4k ..
        const uint32_t H = word(32 + 8 * h + k);  // qh bytes 32h + 4k ..
        g1 = __dp4a(static_cast<int>((A & m4) | ((H << 4) & m2)), xs[0][kk], g1);
        g2 = __dp4a(static_cast<int>((B & m4) | ((H << 2) & m2)), xs[1][kk], g2);
        g3 = __dp4a(static_cast<int>(((A >> 4) & m4) | (H & m2)), xs[2][kk], g3);
        g4 = __dp4a(static_cast<int>(((B >> 4) & m4) | ((H >> 2) & m2)), xs[3][kk], g4);
      }
      const int gs[4] = {g1, g2, g3, g4};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int g = 8 * h + half + 2 * t;
        const int sc = static_cast<int>(static_cast<int8_t>((scw[g >> 2] >> (8 * (g & 3))) & 0xFF));
        const int bsum = (g & 1) ? hi16(a.bs(g >> 1)) : lo16(a.bs(g >> 1));
        sumi += sc * (gs[t] - 32 * bsum);
      }
    }
  }
  const float d = half_bits_to_float(word(52));
  return __fmul_rn(__fmul_rn(d, a.yd()), static_cast<float>(sumi));
}

// Dot of one staged row with the activation: lane g of the row's G lanes
// takes super-block g; the result is valid in all G lanes.
template <class View>
__device__ __forceinline__ float row_dot3v(const uint8_t* row, int type, int g, int G, const View& a) {
  float v = type == NH_TYPE_Q4_K ? sb_dot_q4k3(row + g * kQ4KBytes, a) : sb_dot_q6k3(row + g * kQ6KBytes, a);
  for (int o = 1; o < G; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float row_dot3(const uint8_t* row, int type, int g, int G, const Act3& a) {
  return row_dot3v(row, type, g, G, Act3Regs{a});
}

// Shapes the lane-per-super-block engine covers: K a multiple of 256 with a
// power-of-two count of at most kMaxG super-blocks.
__host__ __device__ inline bool rowdot3_k_ok(int K) {
  if (K < QK || K % QK != 0) return false;
  const int n = K / QK;
  return n <= kMaxG && (n & (n - 1)) == 0;
}

}  // namespace nh

// Batched greedy decode: B independent sequences advanced one position per
// step in lockstep (configuration 3 of the benchmarks: 64 sequences).
//
// Per token the arithmetic is exactly that of the batch-1 kernels (the same
// Q8_K quantisation, super-block dots and butterfly tree, attention splits,
// softmax, top-k and top-k-order combine), so every sequence's ids equal
// those of a batch-1 decode of it.  What changes is the work layout:
//  * activations are prepared once per token (RMS, norm weight, Q8_K) into a
//    global Q8 buffer by batch_prep_kernel, instead of once per CTA;
//  * one grouped row-dot kernel serves QKV, the output projection, the
//    per-expert gate/up and down projections (each expert over the list of
//    tokens routed to it) and lm_head: a warp pass covers 32/G rows x one
//    token, the Q4_K weight super-block stays in registers while the warp
//    walks the CTA's tokens, and the tokens' Q8_K blocks are staged in
//    shared memory;
//  * QK-norm, RoPE and the KV append run once per sequence, then attention
//    runs over (head, 64-position split, sequence) CTAs.
//
// Q8 global block layout (kQ8Stride bytes per 256 values): int8 qs[256] in
// element order, int16 bsums[16], f32 d, padding.
#include <climits>
#include <cstring>

#include "launch.cuh"
#include "rowdot3.cuh"

namespace nh {

constexpr int kQ8Stride = 304;
constexpr int kBatchWarps = 8;
constexpr int kBatchTokTile = 32;  // tokens staged per CTA
constexpr int kBMaxTopK = 32;

// ---------------------------------------------------------------- embed
// Dequantises one embedding row (the element formulas of the batch-1
// embedding, dequantize_row_*) into out[0..n_embd), block-strided.
__device__ __forceinline__ void embed_row(const uint8_t* row, int type, int n_embd, float* out) {
  for (int i = threadIdx.x; i < n_embd; i += blockDim.x) {
    if (type == NH_TYPE_F32) {
      out[i] = reinterpret_cast<const float*>(row)[i];
    } else {
      const int64_t blk = i / QK;
      const int e = i % QK;
      if (type == NH_TYPE_Q4_K) {
        const uint8_t* q = row + blk * kQ4KBytes;
        const float d = half_bits_to_float(q[0] | (q[1] << 8));
        const float dmin = half_bits_to_float(q[2] | (q[3] << 8));
        const int j = e / 32, c = j / 2;
        int sc, m;
        q4k_scale_min(q + 4, j, sc, m);
        const uint8_t byte = q[16 + 32 * c + (e % 32)];
        const int v = (j & 1) ? (byte >> 4) : (byte & 15);
        out[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(v)),
                           __fmul_rn(dmin, static_cast<float>(m)));
      } else {
        const uint8_t* q = row + blk * kQ6KBytes;
        const float d = half_bits_to_float(q[208] | (q[209] << 8));
        const int hh = e / 128, ee = e % 128;
        const int lo = ee < 64 ? (q[64 * hh + ee] & 15) : (q[64 * hh + ee - 64] >> 4);
        const int hi = (q[128 + 32 * hh + ee % 32] >> (2 * (ee / 32))) & 3;
        const int v = (lo | (hi << 4)) - 32;
        const int8_t sc = static_cast<int8_t>(q[192 + e / 16]);
        out[i] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(v));
      }
    }
  }
}

__global__ void batch_embed_kernel(const NhDecodeState* state, const int32_t* prompts, int n_prompt,
                                   const int32_t* fed, const uint8_t* table, int type, int n_embd, int n_vocab,
                                   uint64_t rb, float* h) {
  const int b = blockIdx.x;
  __shared__ int s_tok;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    const int pos = state->pos;
    int tok = pos < n_prompt ? prompts[static_cast<int64_t>(b) * n_prompt + pos] : fed[b];
    if (tok < 0 || tok >= n_vocab) {
      atomicCAS(const_cast<int32_t*>(&state->error), 0, NH_E_ARG);
      tok = 0;
    }
    s_tok = tok;
  }
  __syncthreads();
  embed_row(table + static_cast<uint64_t>(s_tok) * rb, type, n_embd, h + static_cast<int64_t>(b) * n_embd);
}

// Row r of h = embedding row of ids[r] (the prompt positions of a prefill).
// Ids outside the vocabulary read row 0 and raise *err (when not null).
// Row r is id i = r % n_tok of sequence r / n_tok, read at ids[seq *
// ids_stride + i].
__global__ void rows_embed_kernel(const int32_t* ids, int n_tok, int64_t ids_stride, const uint8_t* table, int type,
                                  int n_embd, int n_vocab, uint64_t rb, float* h, int32_t* err) {
  const int r = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  int tok = ids[static_cast<int64_t>(r / n_tok) * ids_stride + r % n_tok];
  if (tok < 0 || tok >= n_vocab) {
    if (threadIdx.x == 0 && err != nullptr) atomicCAS(err, 0, NH_E_ARG);
    tok = 0;
  }
  embed_row(table + static_cast<uint64_t>(tok) * rb, type, n_embd, h + static_cast<int64_t>(r) * n_embd);
}

// ---------------------------------------------------------------- prep
// One CTA per token row: x (optionally RMS-normalised and multiplied by
// norm_w) quantised to Q8_K blocks in global memory; xn (optional) receives
// the normalised f32 row.
__global__ void __launch_bounds__(256) batch_prep_kernel(const float* x, int64_t x_stride, const float* norm_w,
                                                         float eps, int do_norm, int K, uint8_t* q8, float* xn) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ double red[48];
  ActSmem a = carve_act(smem, K, true, norm_w != nullptr && do_norm);
  act_load_norm(a, do_norm ? norm_w : nullptr);
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  prep_act(a, x + r * x_stride, norm_w != nullptr, do_norm != 0, eps, q8 != nullptr, red);
  const int nb = K / QK;
  if (q8 != nullptr) {
    uint8_t* dst = q8 + static_cast<int64_t>(r) * nb * kQ8Stride;
    for (int i = threadIdx.x; i < nb * QK; i += blockDim.x) {
      const int b = i / QK, L = i % QK;
      dst[b * kQ8Stride + L] = static_cast<uint8_t>(a.qs[q8_off(b, L)]);
    }
    for (int i = threadIdx.x; i < nb * 16; i += blockDim.x)
      reinterpret_cast<int16_t*>(dst + (i / 16) * kQ8Stride + 256)[i % 16] = a.bsums[i];
    for (int b = threadIdx.x; b < nb; b += blockDim.x) *reinterpret_cast<float*>(dst + b * kQ8Stride + 288) = a.d[b];
  }
  if (xn != nullptr)
    for (int i = threadIdx.x; i < K; i += blockDim.x) xn[static_cast<int64_t>(r) * K + i] = a.xf[i];
}

// ---------------------------------------------------------------- grouped row dots
// Super-block dots against a Q8 block in shared memory (element-order quants,
// 16-byte loads).  Q4_K: the weight super-block is held in registers.
struct WQ4 {
  uint4 hdr;
  uint4 q[8];
};

__device__ __forceinline__ void load_wq4(WQ4& w, const uint8_t* blk) {
  const uint4* p = reinterpret_cast<const uint4*>(blk);
  w.hdr = __ldg(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) w.q[i] = __ldg(p + 1 + i);
}

__device__ __forceinline__ float dot_q4k_w(const WQ4& w, const uint8_t* ab) {
  const uint32_t sc0 = w.hdr.y & 0x3F3F3F3Fu;
  const uint32_t m0 = w.hdr.z & 0x3F3F3F3Fu;
  const uint32_t sc1 = (w.hdr.w & 0x0F0F0F0Fu) | ((w.hdr.y >> 2) & 0x30303030u);
  const uint32_t m1 = ((w.hdr.w >> 4) & 0x0F0F0F0Fu) | ((w.hdr.z >> 2) & 0x30303030u);
  const uint32_t m4 = 0x0F0F0F0Fu;
  int sumi = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int4 xa = *reinterpret_cast<const int4*>(ab + 64 * c);
    const int4 xb = *reinterpret_cast<const int4*>(ab + 64 * c + 16);
    const int4 xc = *reinterpret_cast<const int4*>(ab + 64 * c + 32);
    const int4 xd = *reinterpret_cast<const int4*>(ab + 64 * c + 48);
    const uint4 w0 = w.q[2 * c], w1 = w.q[2 * c + 1];
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
    const uint32_t scw = c < 2 ? sc0 : sc1;
    sumi += byte_of(scw, (2 * c) & 3) * lo + byte_of(scw, (2 * c + 1) & 3) * hi;
  }
  const int4 bs0 = *reinterpret_cast<const int4*>(ab + 256);
  const int4 bs1 = *reinterpret_cast<const int4*>(ab + 272);
  const int bsw[8] = {bs0.x, bs0.y, bs0.z, bs0.w, bs1.x, bs1.y, bs1.z, bs1.w};
  int summ = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) summ += byte_of(j < 4 ? m0 : m1, j & 3) * (lo16(bsw[j]) + hi16(bsw[j]));
  const float yd = *reinterpret_cast<const float*>(ab + 288);
  const float d = half_bits_to_float(w.hdr.x), dmin = half_bits_to_float(w.hdr.x >> 16);
  return __fsub_rn(__fmul_rn(__fmul_rn(d, yd), static_cast<float>(sumi)),
                   __fmul_rn(__fmul_rn(dmin, yd), static_cast<float>(summ)));
}

// Q6_K: the weight super-block (2-byte aligned, global memory, L1 cached)
// against a shared Q8 block.
__device__ __forceinline__ float dot_q6k_g(const uint8_t* blk, const uint8_t* ab) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(addr & ~static_cast<uintptr_t>(3));
  const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;
  auto word = [&](int i) { return __funnelshift_r(__ldg(base + i), __ldg(base + i + 1), sh); };
  const int* x = reinterpret_cast<const int*>(ab);
  const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
  const uint32_t scw[4] = {word(48), word(49), word(50), word(51)};
  const int4 bs0 = *reinterpret_cast<const int4*>(ab + 256);
  const int4 bs1 = *reinterpret_cast<const int4*>(ab + 272);
  const int bsw[8] = {bs0.x, bs0.y, bs0.z, bs0.w, bs1.x, bs1.y, bs1.z, bs1.w};
  int sumi = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      int g1 = 0, g2 = 0, g3 = 0, g4 = 0;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int k = 4 * half + kk;
        const uint32_t A = word(16 * h + k), B = word(16 * h + 8 + k), H = word(32 + 8 * h + k);
        g1 = __dp4a(static_cast<int>((A & m4) | ((H << 4) & m2)), x[32 * h + k], g1);
        g2 = __dp4a(static_cast<int>((B & m4) | ((H << 2) & m2)), x[32 * h + 8 + k], g2);
        g3 = __dp4a(static_cast<int>(((A >> 4) & m4) | (H & m2)), x[32 * h + 16 + k], g3);
        g4 = __dp4a(static_cast<int>(((B >> 4) & m4) | ((H >> 2) & m2)), x[32 * h + 24 + k], g4);
      }
      const int gs[4] = {g1, g2, g3, g4};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int g = 8 * h + half + 2 * t;
        const int sc = static_cast<int>(static_cast<int8_t>((scw[g >> 2] >> (8 * (g & 3))) & 0xFF));
        const int bsum = (g & 1) ? hi16(bsw[g >> 1]) : lo16(bsw[g >> 1]);
        sumi += sc * (gs[t] - 32 * bsum);
      }
    }
  }
  const float yd = *reinterpret_cast<const float*>(ab + 288);
  return __fmul_rn(__fmul_rn(half_bits_to_float(word(52)), yd), static_cast<float>(sumi));
}

// Epilogues of the grouped row-dot kernel.
enum GroupMode : int { kStore = 0, kResidual = 1, kSwiGLU = 2 };

// Work: n_groups groups; group e multiplies matrix e (base + e * mstride,
// `rows` rows of rb bytes; for SwiGLU a second matrix w2 gives the up rows)
// with the tokens j in [off[e], off[e] + cnt[e]): token j reads Q8 activation
// row act_idx[j] and writes out[out_idx[j] * out_stride + row].  Without
// lists (off null) there is one group over tokens 0 .. n_tok-1.
// blockIdx.x = group * row_blocks + row block; blockIdx.y = token tile.
struct GroupArgs {
  const uint8_t* w;
  const uint8_t* w2;
  uint64_t mstride, mstride2;
  int type, type2;
  int K, rows, rows_per_block;
  uint64_t rb, rb2;
  int n_groups, row_blocks;
  const int32_t* off;
  const int32_t* cnt;
  const int32_t* act_idx;
  const int32_t* out_idx;
  int n_tok;
  const uint8_t* q8;  // [activation rows][K/256] blocks of kQ8Stride bytes
  float* out;
  int64_t out_stride;
  int mode;
  int tok_tile;  // tokens staged per CTA (<= kBatchTokTile)
  int32_t* err;  // NH_E_TIMEOUT when a bounded wait expires (may be null)
  int stages;    // batch_mma_staged_kernel: weight stages per warp
};

__global__ void __launch_bounds__(kBatchWarps * 32, 2) batch_rowdot_kernel(const GroupArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];  // [kBatchTokTile][K/256][kQ8Stride]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.K / QK, G = nb, P = 32 / G;
  const int e = blockIdx.x / p.row_blocks, rblk = blockIdx.x % p.row_blocks;
  pdl_wait();
  pdl_trigger();
  const int t_off = p.off != nullptr ? p.off[e] : 0;
  const int t_cnt = p.off != nullptr ? p.cnt[e] : p.n_tok;
  const int t0 = blockIdx.y * p.tok_tile;
  const int nt = min(p.tok_tile, t_cnt - t0);
  if (nt <= 0) return;
  // Stage this tile's activation rows (16-byte copies).
  const int blk_bytes = nb * kQ8Stride, n16 = blk_bytes / 16;
  for (int q = threadIdx.x; q < nt * n16; q += blockDim.x) {
    const int t = q / n16, part = q % n16;
    const int a = p.act_idx != nullptr ? p.act_idx[t_off + t0 + t] : t0 + t;
    reinterpret_cast<uint4*>(smem + t * blk_bytes)[part] =
        reinterpret_cast<const uint4*>(p.q8 + static_cast<int64_t>(a) * blk_bytes)[part];
  }
  __syncthreads();
  const int g = lane % G, r = lane / G;
  const uint8_t* W = p.w + static_cast<uint64_t>(e) * p.mstride;
  const uint8_t* W2 = p.w2 != nullptr ? p.w2 + static_cast<uint64_t>(e) * p.mstride2 : nullptr;
  const int row_beg = rblk * p.rows_per_block;
  const int row_end = min(p.rows, row_beg + p.rows_per_block);
  // Warps take passes of P rows; every pass walks all staged tokens with the
  // lane's weight super-block held in registers (Q4_K).
  for (int row0 = row_beg + warp * P; row0 < row_end; row0 += kBatchWarps * P) {
    const int row = row0 + r;
    const bool live = row < row_end;
    const int rr = live ? row : row_end - 1;
    const uint8_t* sb = W + static_cast<uint64_t>(rr) * p.rb + g * (p.type == NH_TYPE_Q4_K ? kQ4KBytes : kQ6KBytes);
    const uint8_t* sb2 =
        W2 != nullptr ? W2 + static_cast<uint64_t>(rr) * p.rb2 + g * (p.type2 == NH_TYPE_Q4_K ? kQ4KBytes : kQ6KBytes)
                      : nullptr;
    WQ4 wq, wq2;
    if (p.type == NH_TYPE_Q4_K) load_wq4(wq, sb);
    if (sb2 != nullptr && p.type2 == NH_TYPE_Q4_K) load_wq4(wq2, sb2);
    for (int t = 0; t < nt; ++t) {
      const uint8_t* ab = smem + t * blk_bytes + g * kQ8Stride;
      float v = p.type == NH_TYPE_Q4_K ? dot_q4k_w(wq, ab) : dot_q6k_g(sb, ab);
      for (int o = 1; o < G; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
      float v2 = 0.f;
      if (sb2 != nullptr) {
        v2 = p.type2 == NH_TYPE_Q4_K ? dot_q4k_w(wq2, ab) : dot_q6k_g(sb2, ab);
        for (int o = 1; o < G; o <<= 1) v2 = __fadd_rn(v2, __shfl_xor_sync(0xffffffffu, v2, o));
      }
      if (g == 0 && live) {
        const int o = p.out_idx != nullptr ? p.out_idx[t_off + t0 + t] : t0 + t;
        float* dst = p.out + static_cast<int64_t>(o) * p.out_stride + row;
        if (p.mode == kStore) {
          *dst = v;
        } else if (p.mode == kResidual) {
          *dst = __fadd_rn(*dst, v);
        } else {
          // silu(gate) * up, as the batch-1 gate/up kernel forms it.
          const float s = __fdiv_rn(v, __fadd_rn(1.0f, exp_cw(-v)));
          *dst = __fmul_rn(s, v2);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- tensor-core grouped GEMM (Q4_K)
// The same grouped products on the tensor cores: mma.sync m16n8k32 with int8
// operands computes, for 16 weight rows x 8 tokens, the integer dot of one
// 32-value Q4_K sub-block (A = the 4-bit quants, B = the Q8_K activation
// quants).  Q4_K changes its 6-bit scale every 32 values, so each sub-block's
// int32 result is scaled in registers (sumi += sc_j * dot_j, summ from the
// activation's partial sums) before the super-block is formed in f32 exactly
// as the row-dot kernels form it, and super-blocks are combined by the same
// pairwise tree.  The results are therefore identical to the dp4a kernels.
// (A tcgen05 MMA accumulates over all of K in tensor memory; with a new scale
// every 32 values it would have to be read back after every instruction.)
//
// Work: a warp owns one tile of 16 rows of one group and walks that group's
// tokens 8 at a time (blockIdx.y splits the tokens of ungrouped products).
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Pairwise super-block tree, one value at a time: s-th value v (s from 0).
struct SbTree {
  float p, q, o, r;
  __device__ __forceinline__ void add(int s, float v) {
    if ((s & 1) == 0) {
      p = v;
      r = v;
      return;
    }
    const float pair = __fadd_rn(p, v);
    r = pair;
    if ((s & 2) == 0) {
      q = pair;
      return;
    }
    const float quad = __fadd_rn(q, pair);
    r = quad;
    if ((s & 4) == 0) {
      o = quad;
      return;
    }
    r = __fadd_rn(o, quad);
  }
};

// Super-block s of the tile: rows (g, g+8) at w0 / w1 (the super-block's
// 144 bytes, global or shared memory), the activation blocks of tokens g,
// 2*tig and 2*tig+1 at ag / a0p / a1p; the values join tree[row][token].
__device__ __forceinline__ void sb_q4k_mma(const uint8_t* w0, const uint8_t* w1, const uint8_t* ag,
                                           const uint8_t* a0p, const uint8_t* a1p, int tig, int s,
                                           SbTree (&tree)[2][2]) {
  const uint32_t m4 = 0x0F0F0F0Fu;
  {
    const uint4 h0 = *reinterpret_cast<const uint4*>(w0);
    const uint4 h1 = *reinterpret_cast<const uint4*>(w1);
    uint32_t q0[4][2], q1[4][2];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      q0[c][0] = *reinterpret_cast<const uint32_t*>(w0 + 16 + 32 * c + 4 * tig);
      q0[c][1] = *reinterpret_cast<const uint32_t*>(w0 + 16 + 32 * c + 16 + 4 * tig);
      q1[c][0] = *reinterpret_cast<const uint32_t*>(w1 + 16 + 32 * c + 4 * tig);
      q1[c][1] = *reinterpret_cast<const uint32_t*>(w1 + 16 + 32 * c + 16 + 4 * tig);
    }
    // Scales and mins (6 bits, one per byte) of both rows.
    const uint32_t sc0a = h0.y & 0x3F3F3F3Fu, m0a = h0.z & 0x3F3F3F3Fu;
    const uint32_t sc0b = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t m0b = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t sc1a = h1.y & 0x3F3F3F3Fu, m1a = h1.z & 0x3F3F3F3Fu;
    const uint32_t sc1b = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t m1b = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    int sumi[2][2] = {{0, 0}, {0, 0}};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j >> 1;
      const bool hi = (j & 1) != 0;
      const uint32_t a0 = hi ? (q0[c][0] >> 4) & m4 : q0[c][0] & m4;
      const uint32_t a1 = hi ? (q1[c][0] >> 4) & m4 : q1[c][0] & m4;
      const uint32_t a2 = hi ? (q0[c][1] >> 4) & m4 : q0[c][1] & m4;
      const uint32_t a3 = hi ? (q1[c][1] >> 4) & m4 : q1[c][1] & m4;
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(ag + 32 * j + 4 * tig);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(ag + 32 * j + 16 + 4 * tig);
      int d[4];
      mma_s8(d, a0, a1, a2, a3, b0, b1);
      const int s0 = byte_of(j < 4 ? sc0a : sc0b, j & 3), s1 = byte_of(j < 4 ? sc1a : sc1b, j & 3);
      sumi[0][0] += s0 * d[0];
      sumi[0][1] += s0 * d[1];
      sumi[1][0] += s1 * d[2];
      sumi[1][1] += s1 * d[3];
    }
    // summ and the f32 super-block values for the thread's two tokens.
    const uint8_t* at[2] = {a0p, a1p};
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int4 bs0 = *reinterpret_cast<const int4*>(at[t] + 256);
      const int4 bs1 = *reinterpret_cast<const int4*>(at[t] + 272);
      const int bsw[8] = {bs0.x, bs0.y, bs0.z, bs0.w, bs1.x, bs1.y, bs1.z, bs1.w};
      const float yd = *reinterpret_cast<const float*>(at[t] + 288);
      int summ0 = 0, summ1 = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int pair = lo16(bsw[j]) + hi16(bsw[j]);
        summ0 += byte_of(j < 4 ? m0a : m0b, j & 3) * pair;
        summ1 += byte_of(j < 4 ? m1a : m1b, j & 3) * pair;
      }
      const float d0 = half_bits_to_float(h0.x), dmin0 = half_bits_to_float(h0.x >> 16);
      const float d1 = half_bits_to_float(h1.x), dmin1 = half_bits_to_float(h1.x >> 16);
      tree[0][t].add(s, __fsub_rn(__fmul_rn(__fmul_rn(d0, yd), static_cast<float>(sumi[0][t])),
                                  __fmul_rn(__fmul_rn(dmin0, yd), static_cast<float>(summ0))));
      tree[1][t].add(s, __fsub_rn(__fmul_rn(__fmul_rn(d1, yd), static_cast<float>(sumi[1][t])),
                                  __fmul_rn(__fmul_rn(dmin1, yd), static_cast<float>(summ1))));
    }
  }
}

// One 16x8 tile of one Q4_K matrix over K (nsb super-blocks) read from global
// memory: out[r][t] for rows (g, g+8) and tokens (2*tig, 2*tig+1).
__device__ __forceinline__ void tile_q4k_mma(const uint8_t* w_r0, const uint8_t* w_r1, uint64_t rb, int nsb,
                                             const uint8_t* act_g, const uint8_t* act_t0, const uint8_t* act_t1,
                                             int tig, float (&out)[2][2]) {
  (void)rb;
  SbTree tree[2][2];
  for (int s = 0; s < nsb; ++s)
    sb_q4k_mma(w_r0 + s * kQ4KBytes, w_r1 + s * kQ4KBytes, act_g + s * kQ8Stride, act_t0 + s * kQ8Stride,
               act_t1 + s * kQ8Stride, tig, s, tree);
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < 2; ++t) out[r][t] = tree[r][t].r;
}

__device__ __forceinline__ void mma_s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};\n"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Q6_K: mma m16n8k16 per 16-value group (the format's int8 scale changes
// every 16 values): sumi += sc_g * (dot_g - 32 * bsum_g), then
// (d*yd)*sumi per super-block and the pairwise tree, as sb_dot_q6k3 forms it.
// Super-blocks are 210 bytes, so rows start 2-byte aligned: words are
// assembled from aligned loads with funnel shifts.
// Super-block s of the tile (rows at w0 / w1: the super-block's 210 bytes,
// global or shared memory, 2-byte aligned), as sb_q4k_mma.
__device__ __forceinline__ void sb_q6k_mma(const uint8_t* w0, const uint8_t* w1, const uint8_t* ag,
                                           const uint8_t* a0p, const uint8_t* a1p, int tig, int s,
                                           SbTree (&tree)[2][2]) {
  {
    const uint8_t* wr[2] = {w0, w1};
    const uint32_t* base[2];
    uint32_t sh[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uintptr_t addr = reinterpret_cast<uintptr_t>(wr[r]);
      base[r] = reinterpret_cast<const uint32_t*>(addr & ~static_cast<uintptr_t>(3));
      sh[r] = static_cast<uint32_t>(addr & 3) * 8;
    }
    auto word = [&](int r, int i) { return __funnelshift_r(base[r][i], base[r][i + 1], sh[r]); };
    uint32_t scw[2][4];
    float dd[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
      for (int w = 0; w < 4; ++w) scw[r][w] = word(r, 48 + w);
      dd[r] = half_bits_to_float(word(r, 52));
    }
    const uint8_t* at[2] = {a0p, a1p};
    int bsw[2][8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int4 v0 = *reinterpret_cast<const int4*>(at[t] + 256);
      const int4 v1 = *reinterpret_cast<const int4*>(at[t] + 272);
      bsw[t][0] = v0.x; bsw[t][1] = v0.y; bsw[t][2] = v0.z; bsw[t][3] = v0.w;
      bsw[t][4] = v1.x; bsw[t][5] = v1.y; bsw[t][6] = v1.z; bsw[t][7] = v1.w;
    }
    int sumi[2][2] = {{0, 0}, {0, 0}};
#pragma unroll
    for (int gi = 0; gi < 16; ++gi) {
      // This thread's four values of group gi: elements 16*gi + 4*tig .. +3.
      const int e0 = 16 * gi + 4 * tig;
      const int hh = e0 >> 7, ee = e0 & 127;
      const int ql_word = (64 * hh + (ee & 63)) >> 2, ql_shift = (ee >> 6) * 4;
      const int qh_word = (128 + 32 * hh + (ee & 31)) >> 2, qh_shift = 2 * (ee >> 5);
      uint32_t a[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t lo = (word(r, ql_word) >> ql_shift) & 0x0F0F0F0Fu;
        const uint32_t hi = ((word(r, qh_word) >> qh_shift) & 0x03030303u) << 4;
        a[r] = lo | hi;
      }
      const uint32_t b = *reinterpret_cast<const uint32_t*>(ag + 16 * gi + 4 * tig);
      int d[4];
      mma_s8_k16(d, a[0], a[1], b);
      const int sc0 = static_cast<int>(static_cast<int8_t>((scw[0][gi >> 2] >> (8 * (gi & 3))) & 0xFF));
      const int sc1 = static_cast<int>(static_cast<int8_t>((scw[1][gi >> 2] >> (8 * (gi & 3))) & 0xFF));
      const int bs0 = (gi & 1) ? hi16(bsw[0][gi >> 1]) : lo16(bsw[0][gi >> 1]);
      const int bs1 = (gi & 1) ? hi16(bsw[1][gi >> 1]) : lo16(bsw[1][gi >> 1]);
      sumi[0][0] += sc0 * (d[0] - 32 * bs0);
      sumi[0][1] += sc0 * (d[1] - 32 * bs1);
      sumi[1][0] += sc1 * (d[2] - 32 * bs0);
      sumi[1][1] += sc1 * (d[3] - 32 * bs1);
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float yd = *reinterpret_cast<const float*>(at[t] + 288);
#pragma unroll
      for (int r = 0; r < 2; ++r)
        tree[r][t].add(s, __fmul_rn(__fmul_rn(dd[r], yd), static_cast<float>(sumi[r][t])));
    }
  }
}

// One 16x8 tile of one Q6_K matrix over K read from global memory.
__device__ __forceinline__ void tile_q6k_mma(const uint8_t* w_r0, const uint8_t* w_r1, int nsb,
                                             const uint8_t* act_g, const uint8_t* act_t0, const uint8_t* act_t1,
                                             int tig, float (&out)[2][2]) {
  SbTree tree[2][2];
  for (int s = 0; s < nsb; ++s)
    sb_q6k_mma(w_r0 + s * kQ6KBytes, w_r1 + s * kQ6KBytes, act_g + s * kQ8Stride, act_t0 + s * kQ8Stride,
               act_t1 + s * kQ8Stride, tig, s, tree);
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < 2; ++t) out[r][t] = tree[r][t].r;
}

__global__ void __launch_bounds__(kBatchWarps * 32, 2) batch_mma_kernel(const GroupArgs p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int nsb = p.K / QK;
  const int tiles_per_group = (p.rows + 15) / 16;
  const int ctas_per_group = (tiles_per_group + kBatchWarps - 1) / kBatchWarps;
  const int e = blockIdx.x / ctas_per_group;
  const int rt = (blockIdx.x % ctas_per_group) * kBatchWarps + warp;
  const unsigned ph_idx = phase_begin();
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  if (rt >= tiles_per_group) return;
  const int t_off = p.off != nullptr ? p.off[e] : 0;
  const int t_cnt = p.off != nullptr ? p.cnt[e] : p.n_tok;
  if (t_cnt <= 0) return;
  const int row0 = rt * 16 + g, row1 = row0 + 8;
  const int rr0 = min(row0, p.rows - 1), rr1 = min(row1, p.rows - 1);
  const uint8_t* W = p.w + static_cast<uint64_t>(e) * p.mstride;
  const uint8_t* W2 = p.w2 != nullptr ? p.w2 + static_cast<uint64_t>(e) * p.mstride2 : nullptr;
  const int blk_bytes = nsb * kQ8Stride;
  // The tile's rows are one contiguous slab per matrix: start it towards L2
  // in one request, so the per-super-block loads below hit L2 instead of
  // waiting for DRAM one super-block at a time.
  if (lane == 0) {
    const int nrows = min(16, p.rows - rt * 16);
    const uint8_t* s1 = W + static_cast<uint64_t>(rt) * 16 * p.rb;
    const uint64_t n1 = static_cast<uint64_t>(nrows) * p.rb;
    if (((reinterpret_cast<uintptr_t>(s1) | n1) & 15) == 0) prefetch_l2(s1, static_cast<uint32_t>(n1));
    if (W2 != nullptr) {
      const uint8_t* s2 = W2 + static_cast<uint64_t>(rt) * 16 * p.rb2;
      const uint64_t n2 = static_cast<uint64_t>(nrows) * p.rb2;
      if (((reinterpret_cast<uintptr_t>(s2) | n2) & 15) == 0) prefetch_l2(s2, static_cast<uint32_t>(n2));
    }
  }
  // Token tiles of 8: ungrouped products split them over blockIdx.y.
  const int n_tt = (t_cnt + 7) / 8;
  for (int tt = blockIdx.y; tt < n_tt; tt += gridDim.y) {
    const int tbase = tt * 8;
    auto act_row = [&](int t) {
      const int tc = min(tbase + t, t_cnt - 1);
      const int a = p.act_idx != nullptr ? p.act_idx[t_off + tc] : tc;
      return p.q8 + static_cast<int64_t>(a) * blk_bytes;
    };
    const uint8_t* act_g = act_row(g);
    const uint8_t* act_t0 = act_row(2 * tig);
    const uint8_t* act_t1 = act_row(2 * tig + 1);
    float v[2][2], v2[2][2];
    if (p.type == NH_TYPE_Q4_K)
      tile_q4k_mma(W + static_cast<uint64_t>(rr0) * p.rb, W + static_cast<uint64_t>(rr1) * p.rb, p.rb, nsb, act_g,
                   act_t0, act_t1, tig, v);
    else
      tile_q6k_mma(W + static_cast<uint64_t>(rr0) * p.rb, W + static_cast<uint64_t>(rr1) * p.rb, nsb, act_g, act_t0,
                   act_t1, tig, v);
    if (W2 != nullptr) {
      if (p.type2 == NH_TYPE_Q4_K)
        tile_q4k_mma(W2 + static_cast<uint64_t>(rr0) * p.rb2, W2 + static_cast<uint64_t>(rr1) * p.rb2, p.rb2, nsb,
                     act_g, act_t0, act_t1, tig, v2);
      else
        tile_q6k_mma(W2 + static_cast<uint64_t>(rr0) * p.rb2, W2 + static_cast<uint64_t>(rr1) * p.rb2, nsb, act_g,
                     act_t0, act_t1, tig, v2);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = r == 0 ? row0 : row1;
      if (row >= p.rows) continue;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int tok = tbase + 2 * tig + t;
        if (tok >= t_cnt) continue;
        const int o = p.out_idx != nullptr ? p.out_idx[t_off + tok] : tok;
        float* dst = p.out + static_cast<int64_t>(o) * p.out_stride + row;
        if (p.mode == kStore) {
          *dst = v[r][t];
        } else if (p.mode == kResidual) {
          *dst = __fadd_rn(*dst, v[r][t]);
        } else {
          const float gv = v[r][t];
          const float sl = __fdiv_rn(gv, __fadd_rn(1.0f, exp_cw(-gv)));
          *dst = __fmul_rn(sl, v2[r][t]);
        }
      }
    }
    if (tt == static_cast<int>(blockIdx.y)) phase_stamp(2);  // warp 0's first token tile done
  }
  phase_value(6, static_cast<unsigned long long>(n_tt));
  phase_value(7, static_cast<unsigned long long>(t_cnt));
  phase_value(8, static_cast<unsigned long long>(p.rows) << 32 | static_cast<unsigned>(p.K));
  phase_value(10, reinterpret_cast<uintptr_t>(p.w));  // identifies the launch's weight
  phase_end(kPhBatchMma, ph_idx);
}

// The tensor-core form with its operands in shared memory.  Each warp owns a
// 16-row tile (as batch_mma_kernel) and a ring of `stages` shared-memory
// stages: stage = the tile's 16 rows (of each matrix) for one super-block,
// one bulk copy per row (lane = row; Q6_K blocks through their covering
// 16-byte span), completed on the stage's mbarrier, so the copies of the next
// super-blocks are in flight while this one is multiplied.  The 8 tokens of a
// token tile are copied once per tile into shared memory for all warps.  The
// arithmetic is sb_q4k_mma / sb_q6k_mma's, so results equal batch_mma_kernel's.
constexpr int kMmaSlotQ4 = kQ4KBytes;  // 144: Q4_K blocks start 16-byte aligned
// A 210-byte Q6_K block's covering 16-byte span is at most 224 bytes; the
// reader assembles 4-byte words from an aligned base up to 216 bytes past a
// block start that sits up to 14 bytes into the span: 240 bytes per slot.
constexpr int kMmaSlotQ6 = 240;

__host__ __device__ inline int mma_slot_bytes(int type) { return type == NH_TYPE_Q4_K ? kMmaSlotQ4 : kMmaSlotQ6; }

__global__ void __launch_bounds__(kBatchWarps * 32, 2) batch_mma_staged_kernel(const GroupArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int nsb = p.K / QK, S = p.stages;
  const int nmat = p.w2 != nullptr ? 2 : 1;
  const int slot0 = mma_slot_bytes(p.type), slot1 = mma_slot_bytes(p.type2);
  const int bb0 = p.type == NH_TYPE_Q4_K ? kQ4KBytes : kQ6KBytes;
  const int bb1 = p.type2 == NH_TYPE_Q4_K ? kQ4KBytes : kQ6KBytes;
  const int stage_bytes = 16 * (slot0 + (nmat == 2 ? slot1 : 0));
  const int blk_bytes = nsb * kQ8Stride;
  uint8_t* act_s = smem;                                    // [8 tokens][nsb][kQ8Stride]
  uint64_t* abar = reinterpret_cast<uint64_t*>(smem + 8 * blk_bytes);
  uint64_t* wbar = abar + 1 + warp * S;                     // this warp's stage barriers
  uint8_t* ring = smem + ((8 * blk_bytes + 8 * (1 + kBatchWarps * S) + 127) & ~127) +
                  static_cast<size_t>(warp) * S * stage_bytes;
  const int tiles_per_group = (p.rows + 15) / 16;
  const int ctas_per_group = (tiles_per_group + kBatchWarps - 1) / kBatchWarps;
  const int e = blockIdx.x / ctas_per_group;
  const int rt = (blockIdx.x % ctas_per_group) * kBatchWarps + warp;
  const bool has_rows = rt < tiles_per_group;  // warps without rows still meet the CTA barriers
  const uint8_t* W = p.w + static_cast<uint64_t>(e) * p.mstride;
  const uint8_t* W2 = p.w2 != nullptr ? p.w2 + static_cast<uint64_t>(e) * p.mstride2 : nullptr;
  const unsigned ph_idx = phase_begin();
  if (threadIdx.x == 0) mbar_init(abar, 1);
  if (lane == 0)
    for (int i = 0; i < S; ++i) mbar_init(&wbar[i], 1);
  fence_barrier_init();
  __syncthreads();
  // Stage k of this warp's copies: super-block s into ring stage k % S.
  auto issue = [&](int k, int s) {
    const int st = k % S;
    uint32_t len = 0, off = 0;
    const uint8_t* src = nullptr;
    uint8_t* dst = nullptr;
    if (lane < nmat * 16) {
      const int m = lane >> 4, r = lane & 15;
      const int row = min(rt * 16 + r, p.rows - 1);
      const uint8_t* wb = m == 0 ? W + static_cast<uint64_t>(row) * p.rb + s * bb0
                                 : W2 + static_cast<uint64_t>(row) * p.rb2 + s * bb1;
      src = span16(wb, m == 0 ? bb0 : bb1, &len, &off);
      dst = ring + static_cast<size_t>(st) * stage_bytes + (m == 0 ? r * slot0 : 16 * slot0 + r * slot1);
    }
    uint32_t total = len;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (lane == 0) mbar_expect_tx(&wbar[st], total);
    __syncwarp();
    if (lane < nmat * 16) bulk_g2s(dst, src, len, &wbar[st]);
  };
  int k_issued = 0, k_used = 0;  // this warp's stages issued / consumed (all tiles)
  bool failed = false;
  const bool dense = p.off == nullptr;
  // Dense products: the weights do not depend on the previous kernel.
  const int first_tile = blockIdx.y;
  if (dense && has_rows)
    for (int s = 0; s < min(S, nsb); ++s) issue(k_issued++, s);
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  const int t_off = p.off != nullptr ? p.off[e] : 0;
  const int t_cnt = p.off != nullptr ? p.cnt[e] : p.n_tok;
  const int n_tt = (t_cnt + 7) / 8;
  int it_tile = 0;
  PhaseAcc ph;  // waits for the token rows / for weight stages / multiply
  ph.start();
  for (int tt = first_tile; tt < n_tt; tt += gridDim.y, ++it_tile) {
    const int tbase = tt * 8;
    if (has_rows && !(dense && it_tile == 0))
      for (int s = 0; s < min(S, nsb); ++s) issue(k_issued++, s);
    // The tile's 8 activation rows (clamped past the end), once for all warps.
    __syncthreads();  // every warp is done with the previous tile's rows
    if (warp == 0) {
      uint32_t len = 0;
      const uint8_t* src = nullptr;
      if (lane < 8) {
        const int tc = min(tbase + lane, t_cnt - 1);
        const int a = p.act_idx != nullptr ? p.act_idx[t_off + tc] : tc;
        src = p.q8 + static_cast<int64_t>(a) * blk_bytes;
        len = static_cast<uint32_t>(blk_bytes);
      }
      if (lane == 0) mbar_expect_tx(abar, 8u * static_cast<uint32_t>(blk_bytes));
      __syncwarp();
      if (lane < 8) bulk_g2s(act_s + lane * blk_bytes, src, len, abar);
    }
    if (!mbar_wait(abar, static_cast<uint32_t>(it_tile & 1))) failed = true;
    ph.mark(0);
    float v[2][2] = {{0.f, 0.f}, {0.f, 0.f}}, v2[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    if (has_rows) {
      SbTree tree[2][2][2];
      const uint8_t* ag = act_s + g * blk_bytes;
      const uint8_t* a0 = act_s + (2 * tig) * blk_bytes;
      const uint8_t* a1 = act_s + (2 * tig + 1) * blk_bytes;
      for (int s = 0; s < nsb; ++s) {
        const int st = k_used % S;
        if (!mbar_wait(&wbar[st], static_cast<uint32_t>((k_used / S) & 1))) failed = true;
        ++k_used;
        ph.mark(1);
        const uint8_t* stage = ring + static_cast<size_t>(st) * stage_bytes;
        const int r0 = min(rt * 16 + g, p.rows - 1), r1 = min(rt * 16 + g + 8, p.rows - 1);
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (m >= nmat) break;
          const uint8_t* wm = m == 0 ? W : W2;
          const uint64_t rb = m == 0 ? p.rb : p.rb2;
          const int bb = m == 0 ? bb0 : bb1, sl = m == 0 ? slot0 : slot1;
          const uint8_t* base = stage + (m == 0 ? 0 : 16 * slot0);
          // Offsets of the two rows' blocks inside their 16-byte spans.
          const uint32_t o0 =
              static_cast<uint32_t>(reinterpret_cast<uintptr_t>(wm + static_cast<uint64_t>(r0) * rb + s * bb) & 15);
          const uint32_t o1 =
              static_cast<uint32_t>(reinterpret_cast<uintptr_t>(wm + static_cast<uint64_t>(r1) * rb + s * bb) & 15);
          const uint8_t* w0 = base + (r0 - rt * 16) * sl + o0;
          const uint8_t* w1 = base + (r1 - rt * 16) * sl + o1;
          const int type = m == 0 ? p.type : p.type2;
          if (type == NH_TYPE_Q4_K)
            sb_q4k_mma(w0, w1, ag + s * kQ8Stride, a0 + s * kQ8Stride, a1 + s * kQ8Stride, tig, s, tree[m]);
          else
            sb_q6k_mma(w0, w1, ag + s * kQ8Stride, a0 + s * kQ8Stride, a1 + s * kQ8Stride, tig, s, tree[m]);
        }
        __syncwarp();
        if (s + S < nsb) issue(k_issued++, s + S);
        ph.mark(2);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          v[r][t] = tree[0][r][t].r;
          v2[r][t] = tree[1][r][t].r;
        }
      const int row0 = rt * 16 + g, row1 = row0 + 8;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = r == 0 ? row0 : row1;
        if (row >= p.rows) continue;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int tok = tbase + 2 * tig + t;
          if (tok >= t_cnt) continue;
          const int o = p.out_idx != nullptr ? p.out_idx[t_off + tok] : tok;
          float* dst = p.out + static_cast<int64_t>(o) * p.out_stride + row;
          if (p.mode == kStore) {
            *dst = v[r][t];
          } else if (p.mode == kResidual) {
            *dst = __fadd_rn(*dst, v[r][t]);
          } else {
            const float gv = v[r][t];
            const float sl = __fdiv_rn(gv, __fadd_rn(1.0f, exp_cw(-gv)));
            *dst = __fmul_rn(sl, v2[r][t]);
          }
        }
      }
    }
  }
  // Copies issued for a tile that never started (dense prefetch with no
  // token tile for this CTA) must land before the CTA exits.
  while (k_used < k_issued) {
    if (!mbar_wait(&wbar[k_used % S], static_cast<uint32_t>((k_used / S) & 1))) failed = true;
    ++k_used;
  }
  if (failed && lane == 0 && p.err != nullptr) atomicCAS(p.err, 0, NH_E_TIMEOUT);
  ph.store();
  phase_value(6, static_cast<unsigned long long>(n_tt));
  phase_value(7, static_cast<unsigned long long>(t_cnt));
  phase_value(8, static_cast<unsigned long long>(p.rows) << 32 | static_cast<unsigned>(p.K));
  phase_value(10, reinterpret_cast<uintptr_t>(p.w));
  phase_end(kPhBatchMmaStaged, ph_idx);
}

// ---------------------------------------------------------------- QK-norm, RoPE, KV append
// One CTA per sequence: QK-norm over the full q (and k) width, NEOX RoPE at
// the shared position, the rotated q to qr, and the new K (rotated) and V
// rows appended to the sequence's cache ([B][max_seq][n_embd_kv] per layer).
//
// Row b is position base + b % rows_per_seq (base = state->pos, or pos0 when
// state is null) of cache sequence b / rows_per_seq: decode rows are
// independent sequences at the shared cursor (rows_per_seq 1); prefill rows
// are runs of rows_per_seq consecutive positions, one run per sequence.
__global__ void __launch_bounds__(128) batch_qk_kernel(const NhDecodeState* state, const float* q, const float* k,
                                                       const float* v, const float* q_norm, const float* k_norm,
                                                       float eps, int n_head, int n_head_kv, int hd,
                                                       const float* rope_cs, float* k_cache, float* v_cache,
                                                       int max_seq, float* qr, int pos0, int rows_per_seq) {
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const int dq = n_head * hd, dkv = n_head_kv * hd, half = hd / 2;
  __shared__ double red[16];
  pdl_wait();
  pdl_trigger();
  const int pos = (state != nullptr ? state->pos : pos0) + b % rows_per_seq;
  const int64_t seq = b / rows_per_seq;
  extern __shared__ __align__(16) float qk_s[];  // [dq] q row, [dkv] k row
  copy_to_smem(qk_s, q + static_cast<int64_t>(b) * dq, dq);
  copy_to_smem(qk_s + dq, k + static_cast<int64_t>(b) * dkv, dkv);
  __syncthreads();
  const float* qb = qk_s;
  const float* kb = qk_s + dq;
  double sq = 0.0, sk = 0.0;
  for (int i = tid; i < dq; i += blockDim.x) sq += static_cast<double>(__fmul_rn(qb[i], qb[i]));
  for (int i = tid; i < dkv; i += blockDim.x) sk += static_cast<double>(__fmul_rn(kb[i], kb[i]));
  sq = warp_sum_d(sq);
  sk = warp_sum_d(sk);
  if (lane == 0) {
    red[warp] = sq;
    red[8 + warp] = sk;
  }
  __syncthreads();
  double tq = 0.0, tk = 0.0;
  for (int w = 0; w < nw; ++w) {
    tq += red[w];
    tk += red[8 + w];
  }
  const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(div_count(tq, dq)), eps)));
  const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(div_count(tk, dkv)), eps)));
  const float* cs = rope_cs + static_cast<int64_t>(pos) * hd;
  float* qo = qr + static_cast<int64_t>(b) * dq;
  for (int j = tid; j < n_head * half; j += blockDim.x) {
    const int h = j / half, i = j % half;
    const float c = cs[2 * i], s = cs[2 * i + 1];
    const float x0 = __fmul_rn(__fmul_rn(qb[h * hd + i], scq), q_norm[h * hd + i]);
    const float x1 = __fmul_rn(__fmul_rn(qb[h * hd + i + half], scq), q_norm[h * hd + i + half]);
    qo[h * hd + i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    qo[h * hd + i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
  float* kd = k_cache + (seq * max_seq + pos) * dkv;
  float* vd = v_cache + (seq * max_seq + pos) * dkv;
  for (int j = tid; j < n_head_kv * half; j += blockDim.x) {
    const int h = j / half, i = j % half;
    const float c = cs[2 * i], s = cs[2 * i + 1];
    const float x0 = __fmul_rn(__fmul_rn(kb[h * hd + i], sck), k_norm[h * hd + i]);
    const float x1 = __fmul_rn(__fmul_rn(kb[h * hd + i + half], sck), k_norm[h * hd + i + half]);
    kd[h * hd + i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    kd[h * hd + i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
  const float* vb = v + static_cast<int64_t>(b) * dkv;
  for (int i = tid; i < dkv; i += blockDim.x) vd[i] = vb[i];
}

// ---------------------------------------------------------------- attention
constexpr int kBAttnThreads = 128;
constexpr int kBAttnSplit = 64;

// The thread-per-position score of the batch-1 attention kernel (the same
// lane-strided sums and butterfly tree).
__device__ __forceinline__ float bscore_thread(const float* kr, const float* q, int hd) {
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

struct BAttnArgs {
  NhDecodeState* state;
  const float* qr;
  const float* k_cache;
  const float* v_cache;
  int n_head, n_head_kv, hd, max_seq, n_split;
  float kq_scale;
  unsigned* tickets;  // [B][n_head]
  double* part_l;     // [B][n_head][n_split]
  float* part_m;
  float* part_acc;    // [B][n_head][n_split][hd]
  float* out;         // [B][n_head*hd]
};

__global__ void __launch_bounds__(kBAttnThreads) batch_attention_kernel(const BAttnArgs p) {
  const int h = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int pos = *reinterpret_cast<volatile const int*>(&p.state->pos);
  const int n_kv = pos + 1;
  const int n_active = (n_kv + kBAttnSplit - 1) / kBAttnSplit;
  if (sp >= n_active) return;
  const unsigned ph_idx = phase_begin();
  extern __shared__ __align__(128) float sm[];
  const int hd = p.hd, kst = hd + 4;
  float* Ks = sm;
  float* Vs = Ks + kBAttnSplit * kst;
  float* qh = Vs + kBAttnSplit * hd;
  float* sc = qh + hd;
  __shared__ __align__(8) uint64_t bar;
  __shared__ double red[8];
  __shared__ float s_max[4];
  __shared__ bool s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  const int kh = h / (p.n_head / p.n_head_kv);
  const int dq = p.n_head * hd, dkv = p.n_head_kv * hd;
  const int p0 = sp * kBAttnSplit;
  const int n = min(n_kv, p0 + kBAttnSplit) - p0;
  const uint32_t row = static_cast<uint32_t>(hd) * 4;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  phase_stamp(1);
  pdl_trigger();
  // Every row of the range, including the current position, is in the cache.
  if (tid == 0) mbar_expect_tx(&bar, 2u * row * static_cast<uint32_t>(n));
  __syncthreads();
  {
    const int j = tid & (kBAttnSplit - 1);
    if (j < n) {
      const int64_t g = (static_cast<int64_t>(b) * p.max_seq + p0 + j) * dkv + kh * hd;
      if (tid < kBAttnSplit) bulk_g2s(Ks + j * kst, p.k_cache + g, row, &bar);
      else bulk_g2s(Vs + j * hd, p.v_cache + g, row, &bar);
    }
  }
  copy_to_smem(qh, p.qr + static_cast<int64_t>(b) * dq + h * hd, hd);
  const bool ok = mbar_wait(&bar, 0);
  if (!ok && tid == 0) atomicCAS(&p.state->error, 0, NH_E_TIMEOUT);
  __syncthreads();
  phase_stamp(2);
  float my = -INFINITY;
  if ((hd & 31) == 0) {
    if (tid < n) {
      const float d = bscore_thread(Ks + tid * kst, qh, hd);
      my = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
    }
  } else {
    for (int j = warp; j < n; j += nw) {
      float d = 0.f;
      for (int i = lane; i < hd; i += 32) d = __fadd_rn(d, __fmul_rn(Ks[j * kst + i], qh[i]));
      d = warp_sum(d);
      if (lane == 0) sc[j] = ok ? __fmul_rn(d, p.kq_scale) : 0.f;
    }
    __syncthreads();
    if (tid < n) my = sc[tid];
  }
  float m = warp_max(my);
  if (lane == 0) s_max[warp] = m;
  __syncthreads();
  m = s_max[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, s_max[w]);
  const float e = tid < n ? exp_cw(__fsub_rn(my, m)) : 0.f;
  double l = warp_sum_d(tid < n ? static_cast<double>(e) : 0.0);
  if (lane == 0) red[warp] = l;
  __syncthreads();
  l = 0.0;
  for (int w = 0; w < nw; ++w) l += red[w];
  if (tid < n) sc[tid] = n_active == 1 ? __fmul_rn(e, static_cast<float>(1.0 / l)) : e;
  __syncthreads();
  phase_stamp(3);
  phase_value(6, static_cast<unsigned long long>(n_active));
  float* out = p.out + static_cast<int64_t>(b) * dq + h * hd;
  if (n_active == 1) {
    for (int i = tid; i < hd; i += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < n; ++j) acc = __fadd_rn(acc, __fmul_rn(Vs[j * hd + i], sc[j]));
      out[i] = acc;
    }
    phase_end_sync(kPhBatchAttention, ph_idx);
    return;
  }
  const int64_t bh = static_cast<int64_t>(b) * p.n_head + h;
  const int64_t slot = bh * p.n_split + sp;
  for (int i = tid; i < hd; i += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < n; ++j) acc = __fadd_rn(acc, __fmul_rn(Vs[j * hd + i], sc[j]));
    p.part_acc[slot * hd + i] = acc;
  }
  if (tid == 0) {
    p.part_m[slot] = m;
    p.part_l[slot] = l;
  }
  __syncthreads();
  phase_stamp(4);
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&p.tickets[bh], 1u) == static_cast<unsigned>(n_active - 1);
  }
  __syncthreads();
  phase_stamp(5);
  if (!s_last) {
    phase_end(kPhBatchAttention, ph_idx);
    return;
  }
  phase_value(7, 1);
  __threadfence();
  // The staged K and V rows are no longer read: they hold the split weights
  // and sums (up to 64*(hd+4) floats / 32*hd doubles).
  if (n_active <= kBAttnSplit * kst && n_active <= (kBAttnSplit / 2) * hd) {
    combine_splits(p.part_m + bh * p.n_split, p.part_l + bh * p.n_split, p.part_acc + bh * p.n_split * hd,
                   n_active, hd, Ks, reinterpret_cast<double*>(Vs), out, tid, blockDim.x, true);
    if (tid == 0) p.tickets[bh] = 0u;
    phase_end_sync(kPhBatchAttention, ph_idx);
    return;
  }
  const volatile float* pm = p.part_m + bh * p.n_split;
  const volatile double* pl = p.part_l + bh * p.n_split;
  float M = -INFINITY;
  for (int s = 0; s < n_active; ++s) M = fmaxf(M, pm[s]);
  double L = 0.0;
  for (int s0 = 0; s0 < n_active; s0 += kBAttnSplit) {
    const int cnt = min(kBAttnSplit, n_active - s0);
    __syncthreads();
    for (int s = tid; s < cnt; s += blockDim.x) sc[s] = exp_cw(__fsub_rn(pm[s0 + s], M));
    __syncthreads();
    for (int s = 0; s < cnt; ++s) L += pl[s0 + s] * static_cast<double>(sc[s]);
  }
  const float inv = static_cast<float>(1.0 / L);
  for (int i = tid; i < hd; i += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < n_active; ++s) {
      const float w = exp_cw(__fsub_rn(pm[s], M));
      acc = __fadd_rn(acc, __fmul_rn(__ldcg(&p.part_acc[(bh * p.n_split + s) * hd + i]), w));
    }
    out[i] = __fmul_rn(acc, inv);
  }
  if (tid == 0) p.tickets[bh] = 0u;
  phase_end_sync(kPhBatchAttention, ph_idx);
}

// ---------------------------------------------------------------- prefill attention
// Causal attention of the n_tok prompt positions pos0 .. pos0+n_tok-1 of one
// sequence (query t attends keys 0..pos0+t), with the decode kernels'
// arithmetic for every query: 64-key splits, each with its own maximum,
// exponentials and double sum, combined in split order against the global
// maximum (a single split normalises directly).  A CTA owns kPAttnQ queries
// of one head and walks the splits twice: the first pass finds each query's
// global maximum (scores only), the second re-forms each split and folds it
// into the running combination, so no per-split partials leave the CTA.
constexpr int kPAttnThreads = 256;
constexpr int kPAttnQ = 32;
constexpr int kPAttnSplit = 64;
constexpr int kPAttnGroups = kPAttnThreads / kPAttnSplit;   // query groups (threads per key: one per group)
constexpr int kPAttnPerThread = kPAttnQ / kPAttnGroups;     // queries each thread scores per key
constexpr int kPAttnOut = kPAttnQ * 128 / kPAttnThreads;    // outputs per thread at head_dim 128

// Two queries' scores against one key row with bscore_thread's operation
// order for each (32 lane-strided partial sums over head_dim, then the same
// butterfly), so every score equals bscore_thread(kr, qa/qb) bit for bit;
// each 16-byte chunk of the key row is loaded once for both queries.
__device__ __forceinline__ void bscore_pair(const float* kr, const float* qa, const float* qb, int hd, float& sa,
                                            float& sb) {
  float pa[32], pb[32];
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    pa[l] = 0.f;
    pb[l] = 0.f;
  }
  for (int base = 0; base < hd; base += 32) {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float4 kv = *reinterpret_cast<const float4*>(kr + base + 4 * t);
      const float4 va = *reinterpret_cast<const float4*>(qa + base + 4 * t);
      const float4 vb = *reinterpret_cast<const float4*>(qb + base + 4 * t);
      pa[4 * t + 0] = __fadd_rn(pa[4 * t + 0], __fmul_rn(kv.x, va.x));
      pa[4 * t + 1] = __fadd_rn(pa[4 * t + 1], __fmul_rn(kv.y, va.y));
      pa[4 * t + 2] = __fadd_rn(pa[4 * t + 2], __fmul_rn(kv.z, va.z));
      pa[4 * t + 3] = __fadd_rn(pa[4 * t + 3], __fmul_rn(kv.w, va.w));
      pb[4 * t + 0] = __fadd_rn(pb[4 * t + 0], __fmul_rn(kv.x, vb.x));
      pb[4 * t + 1] = __fadd_rn(pb[4 * t + 1], __fmul_rn(kv.y, vb.y));
      pb[4 * t + 2] = __fadd_rn(pb[4 * t + 2], __fmul_rn(kv.z, vb.z));
      pb[4 * t + 3] = __fadd_rn(pb[4 * t + 3], __fmul_rn(kv.w, vb.w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int l = 0; l < o; ++l) {
      pa[l] = __fadd_rn(pa[l], pa[l + o]);
      pb[l] = __fadd_rn(pb[l], pb[l + o]);
    }
  }
  sa = pa[0];
  sb = pb[0];
}

struct PAttnArgs {
  const float* qr;       // [n_seq][n_tok][n_head*hd] QK-normed, rotated queries
  const float* k_cache;  // [n_seq][max_seq][n_head_kv*hd] post-RoPE keys
  const float* v_cache;
  float* out;            // [n_seq][n_tok][n_head*hd]
  int n_tok, pos0, n_head, n_head_kv, hd, max_seq;
  float kq_scale;
};

__device__ __forceinline__ int pattn_keys_in_split(int n_kv, int s) {
  return max(0, min(kPAttnSplit, n_kv - s * kPAttnSplit));
}

// Grid (head, query block, sequence).
__global__ void __launch_bounds__(kPAttnThreads, 2) prefill_attention_kernel(const PAttnArgs p) {
  const int h = blockIdx.x, t0 = blockIdx.y * kPAttnQ;
  const int nq = min(kPAttnQ, p.n_tok - t0);
  const int hd = p.hd, kst = hd + 4;
  const int kh = h / (p.n_head / p.n_head_kv);
  const int dq = p.n_head * hd, dkv = p.n_head_kv * hd;
  const int64_t row0 = static_cast<int64_t>(blockIdx.z) * p.n_tok;  // the sequence's first row
  const int64_t kv0 = static_cast<int64_t>(blockIdx.z) * p.max_seq * dkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(16) float sm[];
  float* Ks = sm;                      // [64][hd+4]: padded rows for conflict-free 16-byte reads
  float* Vs = Ks + kPAttnSplit * kst;  // [64][hd]
  float* Qs = Vs + kPAttnSplit * hd;   // [kPAttnQ][hd]
  float* S = Qs + kPAttnQ * hd;        // [kPAttnQ][64] scores, then exponentials
  __shared__ float s_max2[2][kPAttnQ];
  __shared__ float s_M[kPAttnQ], s_w[kPAttnQ];
  __shared__ double s_L[kPAttnQ];
  pdl_wait();
  pdl_trigger();
  const int h4 = hd / 4;
  for (int i = tid; i < kPAttnQ * h4; i += blockDim.x) {
    const int q = i / h4, c = i % h4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q < nq) v = reinterpret_cast<const float4*>(p.qr + (row0 + t0 + q) * dq + h * hd)[c];
    reinterpret_cast<float4*>(Qs + q * hd)[c] = v;
  }
  if (tid < kPAttnQ) s_L[tid] = 0.0;
  const int kv_last = p.pos0 + t0 + nq;  // keys the block's last query sees
  const int n_splits = (kv_last + kPAttnSplit - 1) / kPAttnSplit;
  auto n_kv = [&](int q) { return p.pos0 + t0 + q + 1; };
  auto load = [&](int s, bool with_v) {
    const int nk = pattn_keys_in_split(kv_last, s);
    const int64_t r0 = static_cast<int64_t>(s) * kPAttnSplit;
    for (int i = tid; i < nk * h4; i += blockDim.x) {
      const int r = i / h4, c = i % h4;
      const int64_t g = kv0 + (r0 + r) * dkv + kh * hd;
      reinterpret_cast<float4*>(Ks + r * kst)[c] = __ldg(reinterpret_cast<const float4*>(p.k_cache + g) + c);
      if (with_v) reinterpret_cast<float4*>(Vs + r * hd)[c] = __ldg(reinterpret_cast<const float4*>(p.v_cache + g) + c);
    }
  };
  // Scores of the thread's (key j, query q) pairs: j = tid % 64, q = tid / 64
  // + kPAttnGroups * i, two queries per pass over the key row.  Queries past
  // nq read zero rows of Qs; keys past a split's rows are never used.
  const int j = tid & (kPAttnSplit - 1), qh = tid >> 6;
  auto qrow = [&](int i) { return qh + kPAttnGroups * i; };

  // ---- pass 1: each query's maximum over all its keys
  float run[kPAttnPerThread];
#pragma unroll
  for (int i = 0; i < kPAttnPerThread; ++i) run[i] = -INFINITY;
  for (int s = 0; s < n_splits; ++s) {
    __syncthreads();
    load(s, false);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPAttnPerThread; i += 2) {
      const int qa = qrow(i), qb = qrow(i + 1);
      const bool va = qa < nq && j < pattn_keys_in_split(n_kv(qa), s);
      const bool vb = qb < nq && j < pattn_keys_in_split(n_kv(qb), s);
      if (!va && !vb) continue;
      float sa, sb;
      bscore_pair(Ks + j * kst, Qs + qa * hd, Qs + qb * hd, hd, sa, sb);
      if (va) run[i] = fmaxf(run[i], __fmul_rn(sa, p.kq_scale));
      if (vb) run[i + 1] = fmaxf(run[i + 1], __fmul_rn(sb, p.kq_scale));
    }
  }
#pragma unroll
  for (int i = 0; i < kPAttnPerThread; ++i) {
    const float m = warp_max(run[i]);
    if (lane == 0) s_max2[warp & 1][qrow(i)] = m;
  }
  __syncthreads();
  if (tid < kPAttnQ) s_M[tid] = fmaxf(s_max2[0][tid], s_max2[1][tid]);

  // ---- pass 2: form each split and fold it in, in split order
  float acc_out[kPAttnOut];
#pragma unroll
  for (int i = 0; i < kPAttnOut; ++i) acc_out[i] = 0.f;
  const int n_out = kPAttnQ * hd / kPAttnThreads;
  for (int s = 0; s < n_splits; ++s) {
    __syncthreads();
    load(s, true);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPAttnPerThread; i += 2) {
      const int qa = qrow(i), qb = qrow(i + 1);
      const bool va = qa < nq && j < pattn_keys_in_split(n_kv(qa), s);
      const bool vb = qb < nq && j < pattn_keys_in_split(n_kv(qb), s);
      if (!va && !vb) continue;
      float sa, sb;
      bscore_pair(Ks + j * kst, Qs + qa * hd, Qs + qb * hd, hd, sa, sb);
      if (va) S[qa * kPAttnSplit + j] = __fmul_rn(sa, p.kq_scale);
      if (vb) S[qb * kPAttnSplit + j] = __fmul_rn(sb, p.kq_scale);
    }
    __syncthreads();
    // Per query (warp w: queries w, w+4, ...; lane: keys lane and lane+32).
    for (int q = warp; q < nq; q += kPAttnThreads / 32) {
      const int n = pattn_keys_in_split(n_kv(q), s);
      if (n == 0) continue;
      float* sq = S + q * kPAttnSplit;
      const float a = lane < n ? sq[lane] : -INFINITY;
      const float b = lane + 32 < n ? sq[lane + 32] : -INFINITY;
      const float m = warp_max(fmaxf(a, b));
      const float ea = lane < n ? exp_cw(__fsub_rn(a, m)) : 0.f;
      const float eb = lane + 32 < n ? exp_cw(__fsub_rn(b, m)) : 0.f;
      const double la = warp_sum_d(lane < n ? static_cast<double>(ea) : 0.0);
      const double lb = warp_sum_d(lane + 32 < n ? static_cast<double>(eb) : 0.0);
      double l = 0.0;
      l += la;
      l += lb;
      const bool single = n_kv(q) <= kPAttnSplit;
      if (single) {
        const float inv = static_cast<float>(1.0 / l);
        if (lane < n) sq[lane] = __fmul_rn(ea, inv);
        if (lane + 32 < n) sq[lane + 32] = __fmul_rn(eb, inv);
      } else {
        if (lane < n) sq[lane] = ea;
        if (lane + 32 < n) sq[lane + 32] = eb;
        if (lane == 0) {
          const float w = exp_cw(__fsub_rn(m, s_M[q]));
          s_w[q] = w;
          s_L[q] += l * static_cast<double>(w);
        }
      }
    }
    __syncthreads();
#pragma unroll
    for (int it = 0; it < kPAttnOut; ++it) {
      if (it >= n_out) break;
      const int idx = tid + it * kPAttnThreads, q = idx / hd, i = idx % hd;
      if (q >= nq) continue;
      const int n = pattn_keys_in_split(n_kv(q), s);
      if (n == 0) continue;
      const float* sq = S + q * kPAttnSplit;
      float acc = 0.f;
      for (int jj = 0; jj < n; ++jj) acc = __fadd_rn(acc, __fmul_rn(Vs[jj * hd + i], sq[jj]));
      acc_out[it] = n_kv(q) <= kPAttnSplit ? acc : __fadd_rn(acc_out[it], __fmul_rn(acc, s_w[q]));
    }
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < kPAttnOut; ++it) {
    if (it >= n_out) break;
    const int idx = tid + it * kPAttnThreads, q = idx / hd, i = idx % hd;
    if (q >= nq) continue;
    const float v = n_kv(q) <= kPAttnSplit ? acc_out[it] : __fmul_rn(acc_out[it], static_cast<float>(1.0 / s_L[q]));
    p.out[(row0 + t0 + q) * dq + h * hd + i] = v;
  }
}

// ---------------------------------------------------------------- router
// One CTA per token: the E logits from the normalised f32 row (the batch-1
// router's dot order), then softmax and top-(k+1) by rank in warp 0.
//
// With trace_sel/trace_gap, row b is also recorded as the routing of position
// trace_pos0 + b in layer `layer` (the batch-1 router's trace layout).
struct RouterTrace {
  int32_t* sel;
  float* gap;
  int pos0, layer, n_layers;
};

template <int KP>
__global__ void __launch_bounds__(256) batch_router_kernel(const float* xn,
                                                           const float* router, int K, int E, int topk,
                                                           int norm_topk, int32_t* sel, float* wts,
                                                           const RouterTrace tr) {
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float lg[32 * KP];
  __shared__ int s_ids[kBMaxTopK + 1];
  __shared__ float s_vals[kBMaxTopK + 1];
  pdl_wait();
  pdl_trigger();
  const float* x = xn + static_cast<int64_t>(b) * K;
  if (K % 128 == 0 && K <= 2048) {
    // The lane's slice of x stays in registers; each expert row's slice is
    // loaded as one batch before its (ordered) sum.
    constexpr int kV = 2048 / 128;
    float4 xv[kV];
#pragma unroll
    for (int t = 0; t < kV; ++t)
      if (t < K / 128) xv[t] = *reinterpret_cast<const float4*>(x + 4 * lane + 128 * t);
    for (int e = warp; e < E; e += 8) {
      const float4* w4 = reinterpret_cast<const float4*>(router + static_cast<int64_t>(e) * K);
      float4 wv[kV];
#pragma unroll
      for (int t = 0; t < kV; ++t)
        if (t < K / 128) wv[t] = __ldg(w4 + lane + 32 * t);
      float s = 0.f;
#pragma unroll
      for (int t = 0; t < kV; ++t) {
        if (t < K / 128) {
          s = __fadd_rn(s, __fmul_rn(wv[t].x, xv[t].x));
          s = __fadd_rn(s, __fmul_rn(wv[t].y, xv[t].y));
          s = __fadd_rn(s, __fmul_rn(wv[t].z, xv[t].z));
          s = __fadd_rn(s, __fmul_rn(wv[t].w, xv[t].w));
        }
      }
      s = warp_sum(s);
      if (lane == 0) lg[e] = s;
    }
  } else {
    for (int e = warp; e < E; e += 8) {
      const float* w = router + static_cast<int64_t>(e) * K;
      float s = 0.f;
      if (K % 128 == 0) {
        for (int t = 0; t < K / 128; ++t) {
          const float4 wv = *reinterpret_cast<const float4*>(w + 4 * lane + 128 * t);
          const float4 xv = *reinterpret_cast<const float4*>(x + 4 * lane + 128 * t);
          s = __fadd_rn(s, __fmul_rn(wv.x, xv.x));
          s = __fadd_rn(s, __fmul_rn(wv.y, xv.y));
          s = __fadd_rn(s, __fmul_rn(wv.z, xv.z));
          s = __fadd_rn(s, __fmul_rn(wv.w, xv.w));
        }
      } else {
        for (int i = lane; i < K; i += 32) s = __fadd_rn(s, __fmul_rn(w[i], x[i]));
      }
      s = warp_sum(s);
      if (lane == 0) lg[e] = s;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  float pr[KP];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < KP; ++k) {
    const int i = lane + 32 * k;
    pr[k] = i < E ? lg[i] : -INFINITY;
    mx = fmaxf(mx, pr[k]);
  }
  mx = warp_max(mx);
  double sum = 0.0;
#pragma unroll
  for (int k = 0; k < KP; ++k) {
    const int i = lane + 32 * k;
    pr[k] = i < E ? exp_cw(__fsub_rn(pr[k], mx)) : 0.f;
    sum += static_cast<double>(pr[k]);
  }
  sum = warp_sum_d(sum);
  const float inv = static_cast<float>(1.0 / sum);
#pragma unroll
  for (int k = 0; k < KP; ++k) pr[k] = __fmul_rn(pr[k], inv);
  const int kk = min(topk + 1, E);
  int rank[KP];
#pragma unroll
  for (int k = 0; k < KP; ++k) rank[k] = 0;
#pragma unroll
  for (int kj = 0; kj < KP; ++kj) {
#pragma unroll 8
    for (int src = 0; src < 32; ++src) {
      const float pj = __shfl_sync(0xffffffffu, pr[kj], src);
      const int j = src + 32 * kj;
#pragma unroll
      for (int ki = 0; ki < KP; ++ki) {
        const int i = lane + 32 * ki;
        rank[ki] += (j < E && (pj > pr[ki] || (pj == pr[ki] && j < i))) ? 1 : 0;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < KP; ++k) {
    const int i = lane + 32 * k;
    if (i < E && rank[k] < kk) {
      s_ids[rank[k]] = i;
      s_vals[rank[k]] = pr[k];
    }
  }
  __syncwarp();
  float ws = 1.f;
  if (norm_topk) {
    double sw = 0.0;
    for (int t = 0; t < topk; ++t) sw += static_cast<double>(s_vals[t]);
    ws = fmaxf(static_cast<float>(sw), 6.103515625e-5f);
  }
  for (int t = lane; t < topk; t += 32) {
    sel[b * topk + t] = s_ids[t];
    wts[b * topk + t] = norm_topk ? __fdiv_rn(s_vals[t], ws) : s_vals[t];
  }
  if (tr.sel != nullptr) {
    const int64_t rec = static_cast<int64_t>(tr.pos0 + b) * tr.n_layers + tr.layer;
    for (int t = lane; t < topk; t += 32) tr.sel[rec * topk + t] = s_ids[t];
    if (tr.gap != nullptr) {
      // Smallest gap between adjacent probabilities of the descending top-(k+1).
      float g = 1.f;
      for (int t = lane; t + 1 < kk; t += 32) g = fminf(g, __fsub_rn(s_vals[t], s_vals[t + 1]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) g = fminf(g, __shfl_xor_sync(0xffffffffu, g, o));
      if (lane == 0) tr.gap[rec] = g;
    }
  }
}

// ---------------------------------------------------------------- expert plan
// One CTA: for the n_pairs (token, slot) pairs, per-expert counts, offsets and
// the token lists in (token, slot) order: act_idx = token, out_idx = token*k
// + slot.  A stable counting sort: pairs are taken 512 at a time; within a
// chunk a pair's rank among earlier pairs of the same expert is its rank in
// its warp's match set plus the same-expert counts of the earlier warps.
constexpr int kPlanThreads = 512;
constexpr int kPlanWarps = kPlanThreads / 32;

//
// Only experts [e_first, e_first + E) are planned (group e - e_first); pairs
// that selected other experts are left out (expert parallelism: another rank
// owns them).
__global__ void __launch_bounds__(kPlanThreads) batch_moe_plan_kernel(const int32_t* sel, int n_pairs, int e_first,
                                                                      int E, int topk, int32_t* off, int32_t* cnt,
                                                                      int32_t* act_idx, int32_t* out_idx) {
  extern __shared__ int sh[];  // [E] counts, [E] next free index, [kPlanWarps][E] chunk counts
  int* c = sh;
  int* next = sh + E;
  int* wc = sh + 2 * E;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_trigger();
  for (int e = tid; e < E; e += blockDim.x) c[e] = 0;
  for (int i = tid; i < kPlanWarps * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  for (int j = tid; j < n_pairs; j += blockDim.x) {
    const int e = sel[j] - e_first;
    if (e >= 0 && e < E) atomicAdd(&c[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      next[e] = acc;
      acc += c[e];
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    off[e] = next[e];
    cnt[e] = c[e];
  }
  const unsigned lt = (1u << lane) - 1u;
  for (int base = 0; base < n_pairs; base += kPlanThreads) {
    const int j = base + tid;
    const int e = j < n_pairs ? sel[j] - e_first : -1;
    const bool valid = e >= 0 && e < E;
    const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
    const int in_warp = __popc(same & lt);
    if (valid && in_warp == 0) wc[warp * E + e] = __popc(same);
    __syncthreads();
    if (valid) {
      int rank = next[e] + in_warp;
      for (int w = 0; w < warp; ++w) rank += wc[w * E + e];
      act_idx[rank] = j / topk;
      out_idx[rank] = j;
    }
    __syncthreads();
    for (int x = tid; x < E; x += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kPlanWarps; ++w) {
        add += wc[w * E + x];
        wc[w * E + x] = 0;
      }
      next[x] += add;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- expert-parallel combine
// h[b][r] += sum_i wts[b][i] * y_src[b*k+i][r], where y_src is the block that
// the rank owning expert sel[b][i] returned (block = sel / per_rank, blocks
// src_stride floats apart): the batch_combine arithmetic, in top-k order.
__global__ void ep_combine_kernel(const float* y_recv, int64_t src_stride, int n_src, const int32_t* sel,
                                  const float* wts, int topk, int D, int per_rank, float* h) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const float* wb = wts + b * topk;
  const int32_t* sb = sel + b * topk;
  for (int r = blockIdx.y * blockDim.x + threadIdx.x; r < D; r += gridDim.y * blockDim.x) {
    auto y = [&](int i) {
      const int src = min(max(sb[i] / per_rank, 0), n_src - 1);
      return y_recv[static_cast<int64_t>(src) * src_stride + (static_cast<int64_t>(b) * topk + i) * D + r];
    };
    float acc = __fmul_rn(y(0), wb[0]);
    for (int i = 1; i < topk; ++i) acc = __fadd_rn(acc, __fmul_rn(y(i), wb[i]));
    h[static_cast<int64_t>(b) * D + r] = __fadd_rn(h[static_cast<int64_t>(b) * D + r], acc);
  }
}

// ---------------------------------------------------------------- combine
// h[b][r] += sum_i wts[b][i] * y[b*k+i][r], products rounded, added in top-k order.
__global__ void batch_combine_kernel(const float* y, const float* wts, int topk, int D, float* h) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const float* wb = wts + b * topk;
  for (int r = blockIdx.y * blockDim.x + threadIdx.x; r < D; r += gridDim.y * blockDim.x) {
    const float* yb = y + static_cast<int64_t>(b) * topk * D + r;
    float acc = __fmul_rn(yb[0], wb[0]);
    for (int i = 1; i < topk; ++i) acc = __fadd_rn(acc, __fmul_rn(yb[static_cast<int64_t>(i) * D], wb[i]));
    h[static_cast<int64_t>(b) * D + r] = __fadd_rn(h[static_cast<int64_t>(b) * D + r], acc);
  }
}

// ---------------------------------------------------------------- argmax
// One CTA per sequence over its logits (first maximum wins); the last CTA
// advances the shared cursor.
__global__ void batch_argmax_kernel(NhDecodeState* state, const float* logits, int V, int32_t* fed,
                                    int32_t* out_tokens, int n_predict, unsigned* ticket) {
  const int b = blockIdx.x;
  __shared__ float s_bv[32];
  __shared__ int s_bi[32];
  __shared__ bool s_last;
  pdl_wait();
  pdl_trigger();
  const int pos = state->pos, n_prompt = state->n_prompt;
  const bool emit = pos >= n_prompt - 1;
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (emit) {
    const float* lg = logits + static_cast<int64_t>(b) * V;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float v = lg[i];
      if (argmax_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
  }
  block_argmax(bv, bi, s_bv, s_bi);
  if (threadIdx.x == 0) {
    if (emit) {
      if (bi == INT_MAX) bi = 0;
      const int n = pos - (n_prompt - 1);
      if (n < n_predict) out_tokens[static_cast<int64_t>(b) * n_predict + n] = bi;
      fed[b] = bi;
    }
    __threadfence();
    s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (threadIdx.x != 0 || !s_last) return;
  if (emit) state->n_out = state->n_out + 1;
  state->pos = pos + 1;
  *ticket = 0u;
}

}  // namespace nh

using namespace nh;

extern "C" int64_t nh_batch_q8_bytes(int64_t rows, int64_t n) { return rows * (n / QK) * kQ8Stride; }

extern "C" int nh_batch_embed(const NhDecodeState* state, const int32_t* prompts, int n_prompt, const int32_t* fed,
                              int n_seq, const void* table, int32_t type, int64_t n_embd, int64_t n_vocab, float* h,
                              void* stream) {
  if (state == nullptr || prompts == nullptr || fed == nullptr || table == nullptr || h == nullptr || n_seq <= 0)
    return NH_E_ARG;
  if (type != NH_TYPE_F32 && type != NH_TYPE_Q4_K && type != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (type != NH_TYPE_F32 && n_embd % QK != 0) return NH_E_ARG;
  return launch_pdl(batch_embed_kernel, dim3(n_seq), dim3(256), 0, static_cast<cudaStream_t>(stream), state, prompts,
                    n_prompt, fed, static_cast<const uint8_t*>(table), static_cast<int>(type),
                    static_cast<int>(n_embd), static_cast<int>(n_vocab), static_cast<uint64_t>(row_bytes(type, n_embd)),
                    h);
}

extern "C" int nh_batch_prep(const float* x, int64_t x_stride, int64_t rows, const float* norm_w, float eps,
                             int do_norm, int64_t n, void* q8, float* xn, void* stream) {
  if (x == nullptr || rows <= 0 || n <= 0 || n > kMaxK || (q8 == nullptr && xn == nullptr)) return NH_E_ARG;
  if (q8 != nullptr && n % QK != 0) return NH_E_ARG;
  const size_t smem = act_smem_bytes(static_cast<int>(n), true, norm_w != nullptr && do_norm);
  static SmemLimit configured;
  if (!ensure_smem(batch_prep_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(batch_prep_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), smem,
                    static_cast<cudaStream_t>(stream), x, x_stride, norm_w, eps, do_norm, static_cast<int>(n),
                    static_cast<uint8_t*>(q8), xn);
}

// Products of at least this many tokens per call go to the tensor-core form
// (below it the per-CTA token tiles would be mostly empty).
constexpr int kTcMinTokens = 128;


namespace {
// The shared-memory staged form of the tensor-core products is used unless
// NH_MMA_STAGED=0 (read once; both forms give identical results).
bool mma_staged_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = std::getenv("NH_MMA_STAGED");
    v = (s != nullptr && s[0] == '0') ? 0 : 1;
  }
  return v != 0;
}
}  // namespace

extern "C" int nh_batch_rowdot(const NhGroupedRowDot* g, void* stream) {
  if (g == nullptr || g->w == nullptr || g->q8 == nullptr || g->out == nullptr || g->rows <= 0 || g->n_groups <= 0)
    return NH_E_ARG;
  const int eng = g->engine;
  if (eng < NH_ROWDOT_ENGINE_AUTO || eng > NH_ROWDOT_ENGINE_TC) return NH_E_ARG;
  if (eng == NH_ROWDOT_ENGINE_TC ||
      (eng == NH_ROWDOT_ENGINE_AUTO && nh_tc_enabled() && g->max_tokens >= kTcMinTokens)) {
    const int rc = nh_batch_rowdot_tc(g, stream);
    // Outside the tensor-core form's types and shapes (it launched nothing),
    // the automatic choice falls back to the forms below.
    if (rc == NH_OK || eng == NH_ROWDOT_ENGINE_TC || (rc != NH_E_TYPE && rc != NH_E_ARG)) return rc;
  }
  if (!rowdot3_k_ok(static_cast<int>(g->n))) return NH_E_ARG;
  for (int32_t t : {g->type, g->type2})
    if (t != NH_TYPE_Q4_K && t != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (g->mode == kSwiGLU && g->w2 == nullptr) return NH_E_ARG;
  if ((g->type == NH_TYPE_Q4_K && (reinterpret_cast<uintptr_t>(g->w) & 15) != 0) ||
      (g->w2 != nullptr && g->type2 == NH_TYPE_Q4_K && (reinterpret_cast<uintptr_t>(g->w2) & 15) != 0))
    return NH_E_ARG;
  GroupArgs p;
  memset(&p, 0, sizeof(p));
  p.w = static_cast<const uint8_t*>(g->w);
  p.w2 = static_cast<const uint8_t*>(g->w2);
  p.mstride = g->mstride;
  p.mstride2 = g->mstride2;
  p.type = g->type;
  p.type2 = g->w2 != nullptr ? g->type2 : g->type;
  p.K = static_cast<int>(g->n);
  p.rows = static_cast<int>(g->rows);
  p.rb = row_bytes(g->type, g->n);
  p.rb2 = row_bytes(p.type2, g->n);
  p.n_groups = g->n_groups;
  p.off = g->off;
  p.cnt = g->cnt;
  p.act_idx = g->act_idx;
  p.out_idx = g->out_idx;
  p.n_tok = g->n_tok;
  p.q8 = static_cast<const uint8_t*>(g->q8);
  p.out = g->out;
  p.out_stride = g->out_stride;
  p.mode = g->mode;
  p.err = g->err;
  // Work split: row blocks of whole warp passes (8 warps x P rows) and token
  // tiles, aiming at about eight CTAs per SM over all groups so that each
  // warp has only a few passes; smaller token tiles when the row blocks alone
  // cannot get there.
  const int P = 32 / (p.K / QK);
  const int per_pass = kBatchWarps * P;
  const int sms = device_sm_count();
  const int target = std::max(1, 8 * sms / std::max(1, g->n_groups));
  int rpb = (p.rows + target - 1) / target;
  rpb = (rpb + per_pass - 1) / per_pass * per_pass;
  p.rows_per_block = rpb;
  p.row_blocks = (p.rows + rpb - 1) / rpb;
  const int max_tok = std::max(1, g->max_tokens);
  p.tok_tile = kBatchTokTile;
  while (p.tok_tile > 8 && static_cast<int64_t>(p.n_groups) * p.row_blocks * ((max_tok + p.tok_tile - 1) / p.tok_tile) <
                               4 * sms)
    p.tok_tile >>= 1;
  if (eng == NH_ROWDOT_ENGINE_MMA || (eng == NH_ROWDOT_ENGINE_AUTO && batch_mma_enabled())) {
    // Tensor-core form: one warp per 16-row tile; ungrouped products also
    // split their token tiles over grid.y to fill the GPU.
    const int row_tiles = (p.rows + 15) / 16;
    const int ctas_per_group = (row_tiles + kBatchWarps - 1) / kBatchWarps;
    const int tok_tiles = (max_tok + 7) / 8;
    int gy = 1;
    if (p.off == nullptr)
      while (gy < tok_tiles && static_cast<int64_t>(ctas_per_group) * p.n_groups * gy < 4 * sms) ++gy;
    // The staged form copies whole blocks by their 16-byte spans: Q4_K blocks
    // must start 16-byte aligned (span = block), Q6_K blocks 2-byte aligned
    // (span <= 224 bytes), and the activation rows 16-byte aligned.
    auto blocks_ok = [](const void* w, uint64_t mstride, int type) {
      const uintptr_t a = reinterpret_cast<uintptr_t>(w);
      return type == NH_TYPE_Q4_K ? (a & 15) == 0 && (mstride & 15) == 0 : (a & 1) == 0 && (mstride & 1) == 0;
    };
    const bool staged_ok = blocks_ok(p.w, p.mstride, p.type) &&
                           (g->w2 == nullptr || blocks_ok(p.w2, p.mstride2, p.type2)) &&
                           (reinterpret_cast<uintptr_t>(p.q8) & 15) == 0;
    if (staged_ok && mma_staged_enabled()) {
      // Shared-memory operands: the token tile's rows, the barriers and each
      // warp's ring of weight stages (as many as fit two CTAs per SM, 2..4).
      const int nsb = p.K / QK;
      const size_t act = static_cast<size_t>(8) * nsb * kQ8Stride;
      const size_t stage = static_cast<size_t>(16) *
                           (mma_slot_bytes(p.type) + (g->w2 != nullptr ? mma_slot_bytes(p.type2) : 0));
      auto bytes = [&](int S) {
        return ((act + 8 * (1 + kBatchWarps * S) + 127) & ~static_cast<size_t>(127)) +
               static_cast<size_t>(kBatchWarps) * S * stage;
      };
      int S = 4;
      while (S > 2 && bytes(S) > 110 * 1024) --S;
      p.stages = S;
      const size_t smem = bytes(S);
      static SmemLimit configured_staged;
      if (smem <= 220 * 1024 && ensure_smem(batch_mma_staged_kernel, smem, configured_staged)) {
        // Grouped products: a second CTA per (group, row block) takes every
        // other token tile, so experts with many tokens are not walked by one.
        if (p.off != nullptr) gy = std::min(tok_tiles, 2);
        return launch_pdl(batch_mma_staged_kernel, dim3(p.n_groups * ctas_per_group, gy),
                          dim3(kBatchWarps * 32), smem, static_cast<cudaStream_t>(stream), p);
      }
    }
    return launch_pdl(batch_mma_kernel, dim3(p.n_groups * ctas_per_group, gy), dim3(kBatchWarps * 32), 0,
                      static_cast<cudaStream_t>(stream), p);
  }
  const int tiles = (max_tok + p.tok_tile - 1) / p.tok_tile;
  const size_t smem = static_cast<size_t>(p.tok_tile) * (p.K / QK) * kQ8Stride;
  static SmemLimit configured;
  if (!ensure_smem(batch_rowdot_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(batch_rowdot_kernel, dim3(p.n_groups * p.row_blocks, std::max(1, tiles)), dim3(kBatchWarps * 32),
                    smem, static_cast<cudaStream_t>(stream), p);
}

extern "C" int nh_batch_qk(const NhDecodeState* state, const float* q, const float* k, const float* v,
                           const float* q_norm, const float* k_norm, float eps, int n_seq, int n_head, int n_head_kv,
                           int head_dim, const float* rope_cs, float* k_cache, float* v_cache, int max_seq, float* qr,
                           void* stream) {
  if (state == nullptr || q == nullptr || k == nullptr || v == nullptr || q_norm == nullptr || k_norm == nullptr ||
      rope_cs == nullptr || k_cache == nullptr || v_cache == nullptr || qr == nullptr || n_seq <= 0 ||
      head_dim % 2 != 0 || n_head % n_head_kv != 0)
    return NH_E_ARG;
  const size_t smem = static_cast<size_t>(n_head + n_head_kv) * head_dim * sizeof(float);
  static SmemLimit configured;
  if (smem > 220 * 1024 || !ensure_smem(batch_qk_kernel, smem, configured)) return NH_E_ARG;
  return launch_pdl(batch_qk_kernel, dim3(n_seq), dim3(128), smem, static_cast<cudaStream_t>(stream), state, q, k, v,
                    q_norm, k_norm, eps, n_head, n_head_kv, head_dim, rope_cs, k_cache, v_cache, max_seq, qr, 0, 1);
}

extern "C" int64_t nh_batch_attention_scratch_bytes(int n_seq, int n_head, int head_dim, int max_seq) {
  const int64_t S = (max_seq + kBAttnSplit - 1) / kBAttnSplit;
  const int64_t bh = static_cast<int64_t>(n_seq) * n_head;
  return ((bh * 4 + 255) / 256) * 256 + bh * S * (8 + 4 + 4 * static_cast<int64_t>(head_dim)) + 512;
}

extern "C" int nh_batch_attention(const NhDecodeState* state, const float* qr, int n_seq, int n_head, int n_head_kv,
                                  int head_dim, float kq_scale, const float* k_cache, const float* v_cache, int max_seq,
                                  void* scratch, float* out, void* stream) {
  if (state == nullptr || qr == nullptr || k_cache == nullptr || v_cache == nullptr || scratch == nullptr ||
      out == nullptr || n_seq <= 0 || head_dim % 4 != 0 || head_dim > 256 || n_head % n_head_kv != 0 ||
      (reinterpret_cast<uintptr_t>(k_cache) & 15) != 0 || (reinterpret_cast<uintptr_t>(v_cache) & 15) != 0)
    return NH_E_ARG;
  BAttnArgs p;
  p.state = const_cast<NhDecodeState*>(state);
  p.qr = qr;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.n_head = n_head;
  p.n_head_kv = n_head_kv;
  p.hd = head_dim;
  p.max_seq = max_seq;
  p.n_split = (max_seq + kBAttnSplit - 1) / kBAttnSplit;
  p.kq_scale = kq_scale;
  const int64_t bh = static_cast<int64_t>(n_seq) * n_head;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  p.tickets = reinterpret_cast<unsigned*>(sc);
  int64_t off = ((bh * 4 + 255) / 256) * 256;
  p.part_l = reinterpret_cast<double*>(sc + off);
  off += bh * p.n_split * 8;
  p.part_m = reinterpret_cast<float*>(sc + off);
  off += bh * p.n_split * 4;
  off = (off + 15) & ~15ll;
  p.part_acc = reinterpret_cast<float*>(sc + off);
  p.out = out;
  const size_t smem = static_cast<size_t>(kBAttnSplit * (head_dim + 4) + kBAttnSplit * head_dim + head_dim +
                                          kBAttnSplit) * sizeof(float);
  static SmemLimit configured;
  if (!ensure_smem(batch_attention_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(batch_attention_kernel, dim3(n_head, p.n_split, n_seq), dim3(kBAttnThreads), smem,
                    static_cast<cudaStream_t>(stream), p);
}

extern "C" int nh_prefill_embed_seqs(const int32_t* ids, int64_t ids_stride, int n_seq, int n_tok, const void* table,
                                     int32_t type, int64_t n_embd, int64_t n_vocab, float* h, int32_t* err,
                                     void* stream) {
  if (ids == nullptr || table == nullptr || h == nullptr || n_tok <= 0 || n_seq <= 0 ||
      (n_seq > 1 && ids_stride < n_tok) || static_cast<int64_t>(n_seq) * n_tok > INT32_MAX)
    return NH_E_ARG;
  if (type != NH_TYPE_F32 && type != NH_TYPE_Q4_K && type != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (type != NH_TYPE_F32 && n_embd % QK != 0) return NH_E_ARG;
  return launch_pdl(rows_embed_kernel, dim3(n_seq * n_tok), dim3(256), 0, static_cast<cudaStream_t>(stream), ids,
                    n_tok, ids_stride, static_cast<const uint8_t*>(table), static_cast<int>(type),
                    static_cast<int>(n_embd), static_cast<int>(n_vocab),
                    static_cast<uint64_t>(row_bytes(type, n_embd)), h, err);
}

extern "C" int nh_prefill_embed(const int32_t* ids, int n_tok, const void* table, int32_t type, int64_t n_embd,
                                int64_t n_vocab, float* h, int32_t* err, void* stream) {
  return nh_prefill_embed_seqs(ids, n_tok, 1, n_tok, table, type, n_embd, n_vocab, h, err, stream);
}

extern "C" int nh_prefill_qk_seqs(const float* q, const float* k, const float* v, const float* q_norm,
                                  const float* k_norm, float eps, int n_seq, int n_tok, int pos0, int n_head,
                                  int n_head_kv, int head_dim, const float* rope_cs, float* k_cache, float* v_cache,
                                  int max_seq, float* qr, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || q_norm == nullptr || k_norm == nullptr || rope_cs == nullptr ||
      k_cache == nullptr || v_cache == nullptr || qr == nullptr || n_seq <= 0 || n_tok <= 0 || pos0 < 0 ||
      head_dim % 2 != 0 || n_head <= 0 || n_head_kv <= 0 || n_head % n_head_kv != 0 || pos0 + n_tok > max_seq ||
      static_cast<int64_t>(n_seq) * n_tok > INT32_MAX)
    return NH_E_ARG;
  const size_t smem = static_cast<size_t>(n_head + n_head_kv) * head_dim * sizeof(float);
  static SmemLimit configured;
  if (smem > 220 * 1024 || !ensure_smem(batch_qk_kernel, smem, configured)) return NH_E_ARG;
  return launch_pdl(batch_qk_kernel, dim3(n_seq * n_tok), dim3(128), smem, static_cast<cudaStream_t>(stream),
                    static_cast<const NhDecodeState*>(nullptr), q, k, v, q_norm, k_norm, eps, n_head, n_head_kv,
                    head_dim, rope_cs, k_cache, v_cache, max_seq, qr, pos0, n_tok);
}

extern "C" int nh_prefill_qk(const float* q, const float* k, const float* v, const float* q_norm, const float* k_norm,
                             float eps, int n_tok, int pos0, int n_head, int n_head_kv, int head_dim,
                             const float* rope_cs, float* k_cache, float* v_cache, int max_seq, float* qr,
                             void* stream) {
  return nh_prefill_qk_seqs(q, k, v, q_norm, k_norm, eps, 1, n_tok, pos0, n_head, n_head_kv, head_dim, rope_cs,
                            k_cache, v_cache, max_seq, qr, stream);
}

extern "C" int nh_prefill_attention_seqs(const float* qr, int n_seq, int n_tok, int pos0, int n_head, int n_head_kv,
                                         int head_dim, float kq_scale, const float* k_cache, const float* v_cache,
                                         int max_seq, float* out, void* stream) {
  if (qr == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || n_seq <= 0 || n_seq > 65535 ||
      n_tok <= 0 || pos0 < 0 || pos0 + n_tok > max_seq || n_head <= 0 || n_head_kv <= 0 ||
      n_head % n_head_kv != 0 || head_dim % 32 != 0 || head_dim > 128 ||
      (reinterpret_cast<uintptr_t>(k_cache) & 15) != 0 || (reinterpret_cast<uintptr_t>(v_cache) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(qr) & 15) != 0)
    return NH_E_ARG;
  PAttnArgs p;
  p.qr = qr;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.out = out;
  p.n_tok = n_tok;
  p.pos0 = pos0;
  p.n_head = n_head;
  p.n_head_kv = n_head_kv;
  p.hd = head_dim;
  p.max_seq = max_seq;
  p.kq_scale = kq_scale;
  const size_t smem = static_cast<size_t>(kPAttnSplit * (head_dim + 4) + kPAttnSplit * head_dim +
                                          kPAttnQ * head_dim + kPAttnQ * kPAttnSplit) * sizeof(float);
  static SmemLimit configured;
  if (!ensure_smem(prefill_attention_kernel, smem, configured)) return NH_E_CUDA;
  return launch_pdl(prefill_attention_kernel, dim3(n_head, (n_tok + kPAttnQ - 1) / kPAttnQ, n_seq),
                    dim3(kPAttnThreads), smem, static_cast<cudaStream_t>(stream), p);
}

extern "C" int nh_prefill_attention(const float* qr, int n_tok, int pos0, int n_head, int n_head_kv, int head_dim,
                                    float kq_scale, const float* k_cache, const float* v_cache, int max_seq,
                                    float* out, void* stream) {
  return nh_prefill_attention_seqs(qr, 1, n_tok, pos0, n_head, n_head_kv, head_dim, kq_scale, k_cache, v_cache,
                                   max_seq, out, stream);
}

extern "C" int nh_batch_router_trace(const float* xn, const float* router, int n_seq, int64_t n_embd, int n_expert,
                                     int k, int norm_topk, int32_t* sel, float* wts, int32_t* trace_sel,
                                     float* trace_gap, int trace_pos0, int layer, int n_layers, void* stream) {
  if (xn == nullptr || router == nullptr || sel == nullptr || wts == nullptr || n_seq <= 0 || n_expert <= 0 ||
      n_expert > 256 || k <= 0 || k > kBMaxTopK || k > n_expert || n_embd % 4 != 0)
    return NH_E_ARG;
  if (trace_sel != nullptr && (trace_pos0 < 0 || layer < 0 || layer >= n_layers)) return NH_E_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int K = static_cast<int>(n_embd);
  const RouterTrace tr{trace_sel, trace_sel != nullptr ? trace_gap : nullptr, trace_pos0, layer, n_layers};
  if (n_expert <= 32)
    return launch_pdl(batch_router_kernel<1>, dim3(n_seq), dim3(256), 0, st, xn, router, K, n_expert, k, norm_topk,
                      sel, wts, tr);
  if (n_expert <= 64)
    return launch_pdl(batch_router_kernel<2>, dim3(n_seq), dim3(256), 0, st, xn, router, K, n_expert, k, norm_topk,
                      sel, wts, tr);
  if (n_expert <= 128)
    return launch_pdl(batch_router_kernel<4>, dim3(n_seq), dim3(256), 0, st, xn, router, K, n_expert, k, norm_topk,
                      sel, wts, tr);
  return launch_pdl(batch_router_kernel<8>, dim3(n_seq), dim3(256), 0, st, xn, router, K, n_expert, k, norm_topk,
                    sel, wts, tr);
}

extern "C" int nh_batch_router(const float* xn, const float* router, int n_seq, int64_t n_embd, int n_expert, int k,
                               int norm_topk, int32_t* sel, float* wts, void* stream) {
  return nh_batch_router_trace(xn, router, n_seq, n_embd, n_expert, k, norm_topk, sel, wts, nullptr, nullptr, 0, 0, 1,
                               stream);
}

extern "C" int nh_batch_moe_plan_range(const int32_t* sel, int n_seq, int k, int e_first, int n_expert,
                                       int32_t* off, int32_t* cnt, int32_t* act_idx, int32_t* out_idx, void* stream) {
  if (sel == nullptr || off == nullptr || cnt == nullptr || act_idx == nullptr || out_idx == nullptr || n_seq <= 0 ||
      k <= 0 || n_expert <= 0 || e_first < 0)
    return NH_E_ARG;
  const int n_pairs = n_seq * k;
  const size_t smem = static_cast<size_t>(2 + kPlanWarps) * n_expert * sizeof(int);
  if (smem > 48 * 1024) return NH_E_CAPACITY;
  return launch_pdl(batch_moe_plan_kernel, dim3(1), dim3(kPlanThreads), smem, static_cast<cudaStream_t>(stream), sel,
                    n_pairs, e_first, n_expert, k, off, cnt, act_idx, out_idx);
}

extern "C" int nh_batch_moe_plan(const int32_t* sel, int n_seq, int k, int n_expert, int32_t* off, int32_t* cnt,
                                 int32_t* act_idx, int32_t* out_idx, void* stream) {
  return nh_batch_moe_plan_range(sel, n_seq, k, 0, n_expert, off, cnt, act_idx, out_idx, stream);
}

extern "C" int nh_ep_combine(const float* y_recv, int64_t src_stride, int n_src, const int32_t* sel, const float* wts,
                             int n_seq, int k, int64_t n_embd, int experts_per_rank, float* h, void* stream) {
  if (y_recv == nullptr || sel == nullptr || wts == nullptr || h == nullptr || n_seq <= 0 || k <= 0 || n_src <= 0 ||
      experts_per_rank <= 0 || src_stride < static_cast<int64_t>(n_seq) * k * n_embd)
    return NH_E_ARG;
  return launch_pdl(ep_combine_kernel, dim3(n_seq, static_cast<unsigned>((n_embd + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), y_recv, src_stride, n_src, sel, wts, k,
                    static_cast<int>(n_embd), experts_per_rank, h);
}

extern "C" int nh_batch_combine(const float* y, const float* wts, int n_seq, int k, int64_t n_embd, float* h,
                                void* stream) {
  if (y == nullptr || wts == nullptr || h == nullptr || n_seq <= 0 || k <= 0) return NH_E_ARG;
  return launch_pdl(batch_combine_kernel, dim3(n_seq, static_cast<unsigned>((n_embd + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), y, wts, k,
                    static_cast<int>(n_embd), h);
}

extern "C" int nh_batch_argmax(NhDecodeState* state, const float* logits, int n_seq, int64_t n_vocab, int32_t* fed,
                               int32_t* out_tokens, int n_predict, void* scratch, void* stream) {
  if (state == nullptr || logits == nullptr || fed == nullptr || out_tokens == nullptr || scratch == nullptr ||
      n_seq <= 0)
    return NH_E_ARG;
  return launch_pdl(batch_argmax_kernel, dim3(n_seq), dim3(256), 0, static_cast<cudaStream_t>(stream), state, logits,
                    static_cast<int>(n_vocab), fed, out_tokens, n_predict, static_cast<unsigned*>(scratch));
}

NH_PHASE_TRACE_SETTER(batch)

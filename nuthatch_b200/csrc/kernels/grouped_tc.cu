// Grouped Q4_K x Q8_K products on the 5th-generation tensor cores (tcgen05,
// kind::i8, accumulators in tensor memory): ggml_mul_mat_id for batches of
// tokens (moe.cc:41-50) and the dense projections of a prompt prefill.
//
// Exactness.  A Q4_K super-block's value against a Q8_K activation block is
//   (d*yd)*sum_j sc_j*<q4,q8>_j  -  (dmin*yd)*sum_j m_j*(bsum_2j + bsum_2j+1)
// with a new 6-bit scale sc_j every 32 values.  One kind::i8 MMA with K = 32
// covers exactly one 32-value sub-block, so every sub-block's integer dot
// lands in its own tensor-memory accumulator (8 per super-block and matrix,
// each N = 32 token columns wide); the epilogue reads them back once per
// super-block, forms the integer sums in registers, applies d, dmin and the
// activation scale in the order the row-dot kernels use, and adds the
// super-blocks with the same pairwise tree.  Results are identical to the
// dp4a and mma.sync forms bit for bit.
//
// Work.  A CTA owns 128 weight rows (one per tensor-memory lane) of one group
// and 32 of that group's tokens, for one or two matrices (gate and up for
// SwiGLU), over all of K.  Per super-block: the raw Q4_K blocks and the
// tokens' Q8_K blocks arrive by cp.async in a double-buffered staging area
// (the next super-block's copies run during this one's MMAs and epilogue);
// the activation quants land directly in the MMA's K-major core-matrix layout;
// the 4-bit weight quants are widened to int8 into the same layout; one thread
// issues the 8 (or 16) MMAs and commits them to an mbarrier; 8 warps read the
// accumulators (warp w: lanes 32*(w%4).., tokens 16*(w/4)..) and form the
// values.  All waits are bounded; an expired wait records NH_E_TIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "launch.cuh"
#include "rowdot3.cuh"

namespace nh {

namespace {

constexpr int kTcRows = 128;    // weight rows per CTA = tensor-memory lanes
constexpr int kTcTok = 32;      // tokens per CTA = accumulator columns
constexpr int kTcThreads = 256;
constexpr int kTcQ8Stride = 304;  // Q8 activation block: qs[256], sums int16[16], d f32, pad
constexpr int kTcKBlocks = 8;     // 32-value sub-blocks per super-block
constexpr int kTcLdBatch = 4;     // accumulator loads per tensor-memory wait (divides kTcKBlocks)

// Shared-memory layout (bytes from a 1024-aligned base).
constexpr int kAOpBytes = kTcKBlocks * kTcRows * 32;   // one matrix, one super-block: 32 KB
constexpr int kBOpBytes = kTcKBlocks * kTcTok * 32;    // one stage: 8 KB
constexpr int kARawRow = 144;                          // one Q4_K block
constexpr int kARawBytes = kTcRows * kARawRow;         // one matrix, one stage: 18 KB
constexpr int kBMetaBytes = kTcTok * 48;               // sums + scale per token, one stage
constexpr int kOffAOp = 0;
constexpr int kOffBOp = kOffAOp + 2 * kAOpBytes;
constexpr int kOffARaw = kOffBOp + 2 * kBOpBytes;
constexpr int kOffBMeta = kOffARaw + 2 * 2 * kARawBytes;
constexpr int kOffBsp = kOffBMeta + 2 * kBMetaBytes;      // [kTcTok][8] int
constexpr int kOffBar = kOffBsp + kTcTok * 8 * 4;
constexpr int kTcRowTabTiles = 16;                        // token tiles whose rows are tabulated
constexpr int kOffRowTab = kOffBar + 64;                  // [kTcRowTabTiles][kTcTok] activation rows
static_assert(kTcThreads == kTcTok * 8, "one thread per (token, sub-block) sum");
constexpr int kTcSmemBytes = kOffRowTab + kTcRowTabTiles * kTcTok * 4 + 1024;  // + alignment slack

struct TcArgs {
  // Tensor maps of the weights (2-D: row bytes x group rows, boxes of one
  // Q4_K block x kTcRows rows), used when use_tma; else cp.async per row.
  CUtensorMap tmap[2];
  int use_tma;
  const uint8_t* w;
  const uint8_t* w2;
  uint64_t mstride, mstride2, rb;
  int K, rows, row_tiles, mode, n_tok;
  const int32_t* off;
  const int32_t* cnt;
  const int32_t* act_idx;
  const int32_t* out_idx;
  const uint8_t* q8;
  float* out;
  int64_t out_stride;
  int32_t* err;
};

// K-major, no-swizzle core-matrix layout of one 32-byte K block: 8-row
// groups 256 bytes apart, the two 16-byte K chunks of a row 128 bytes apart.
__device__ __forceinline__ uint32_t core_off(int row, int kc) {
  return static_cast<uint32_t>((row >> 3) * 256 + kc * 128 + (row & 7) * 16);
}

// UMMA shared-memory descriptor (K-major, SWIZZLE_NONE): start address,
// leading byte offset (between K chunks) 128, stride byte offset (between
// 8-row groups) 256, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
         (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor: D s32, A s8, B s8, both K-major, N = kTcTok, M = 128.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTcTok >> 3) << 17) |
                            (static_cast<uint32_t>(kTcRows >> 4) << 24);

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(0)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive accumulator columns of the warp's 32 lanes; the registers
// hold them only after tc_wait_ld.
__device__ __forceinline__ void tc_ld16_issue(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// One box of a 2-D tensor map into shared memory, completing on `bar`
// (no multicast).  x is in bytes of the row (a multiple of 16), y the row.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Pairwise super-block tree, one value at a time (the row-dot kernels' order).
struct Tree {
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

template <int NMAT>
__global__ void __launch_bounds__(kTcThreads, 1) grouped_q4k_tc_kernel(const __grid_constant__ TcArgs p) {
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffBar + 16);
  uint64_t* sbar = reinterpret_cast<uint64_t*>(sm + kOffBar + 32);  // [2] weight stages (tensor-map loads)
  int32_t* bsp = reinterpret_cast<int32_t*>(sm + kOffBsp);  // [kTcTok][8] sub-block sums of the activation
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int e = blockIdx.x / p.row_tiles, rt = blockIdx.x % p.row_tiles;
  pdl_wait();
  pdl_trigger();
  const int t_off = p.off != nullptr ? p.off[e] : 0;
  const int t_cnt = p.off != nullptr ? p.cnt[e] : p.n_tok;
  // Token tiles blockIdx.y, blockIdx.y + gridDim.y, ... of this group.
  const int n_tiles = (t_cnt + kTcTok - 1) / kTcTok;
  const int my_tiles = n_tiles > static_cast<int>(blockIdx.y)
                           ? (n_tiles - static_cast<int>(blockIdx.y) + static_cast<int>(gridDim.y) - 1) /
                                 static_cast<int>(gridDim.y)
                           : 0;
  if (my_tiles == 0) return;  // nothing allocated yet
  const unsigned ph_idx = phase_begin();
  PhaseAcc ph;  // wait for the stage / widen / MMA / epilogue, per iteration
  ph.start();
  const int row0 = rt * kTcRows;
  const int nsb = p.K / QK;
  const int total = my_tiles * nsb;  // (tile, super-block) iterations
  constexpr uint32_t kCols = NMAT == 2 ? 512u : 256u;

  auto tile_base = [&](int it) { return (static_cast<int>(blockIdx.y) + (it / nsb) * static_cast<int>(gridDim.y)) * kTcTok; };
  // Activation row of token t of a tile (clamped to the last valid token past
  // the end), from global memory.
  auto act_index = [&](int tok_base, int t) {
    const int tc = min(tok_base + t, t_cnt - 1);
    return p.act_idx != nullptr ? p.act_idx[t_off + tc] : tc;
  };
  // The rows of this CTA's first kTcRowTabTiles tiles, read once here (the
  // barrier after the tensor-memory allocation orders them), so the copies
  // issued per super-block wait on no global load.
  int32_t* row_tab = reinterpret_cast<int32_t*>(sm + kOffRowTab);
  for (int i = tid; i < min(my_tiles, kTcRowTabTiles) * kTcTok; i += kTcThreads) {
    const int k = i / kTcTok;
    row_tab[i] = act_index((static_cast<int>(blockIdx.y) + k * static_cast<int>(gridDim.y)) * kTcTok, i % kTcTok);
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(&sbar[0], 1);
    mbar_init(&sbar[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto act_row = [&](int it, int t) {
    const int k = it / nsb;
    const int a = k < kTcRowTabTiles ? row_tab[k * kTcTok + t] : act_index(tile_base(it), t);
    return p.q8 + static_cast<int64_t>(a) * nsb * kTcQ8Stride;
  };
  const uint8_t* wmat[2] = {p.w + static_cast<uint64_t>(e) * p.mstride,
                            NMAT == 2 ? p.w2 + static_cast<uint64_t>(e) * p.mstride2 : nullptr};

  // Copies of iteration it into stage st: raw weight blocks (thread = row,
  // nine 16-byte chunks), activation quants in MMA layout, activation sums
  // and scale.
  auto issue = [&](int it, int st) {
    const int sb = it % nsb;
    if (p.use_tma) {
      if (tid == 0) {
        // The stage's previous contents were read through the generic proxy
        // (ordered before this thread by the CTA barrier): order them before
        // the tensor-map writes.
        fence_async_smem();
        mbar_expect_tx(&sbar[st], static_cast<uint32_t>(NMAT * kARawBytes));
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
          tma_load_2d(smem_u32(sm + kOffARaw + st * 2 * kARawBytes + m * kARawBytes), &p.tmap[m], sb * kARawRow,
                      e * p.rows + row0, &sbar[st]);
      }
    } else if (tid < NMAT * kTcRows) {
      const int m = tid / kTcRows, r = tid % kTcRows;
      const int row = min(row0 + r, p.rows - 1);
      const uint32_t dst = smem_u32(sm + kOffARaw + st * 2 * kARawBytes + (m * kTcRows + r) * kARawRow);
      const uint8_t* src = wmat[m] + static_cast<uint64_t>(row) * p.rb + sb * kARawRow;
#pragma unroll
      for (int c = 0; c < 9; ++c) cp_async16(dst + c * 16, src + c * 16);
    }
    const uint32_t bop = smem_u32(sm + kOffBOp + st * kBOpBytes);
    const uint32_t bmeta = smem_u32(sm + kOffBMeta + st * kBMetaBytes);
    for (int i = tid; i < kTcTok * 19; i += kTcThreads) {
      const int t = i / 19, c = i - t * 19;
      const uint8_t* src = act_row(it, t) + sb * kTcQ8Stride + c * 16;
      if (c < 16)
        cp_async16(bop + (c >> 1) * (kTcTok * 32) + core_off(t, c & 1), src);
      else
        cp_async16(bmeta + t * 48 + (c - 16) * 16, src);
    }
    cp_async_commit();
  };

  Tree tree[NMAT][16];
  const int q4 = warp & 3, th = warp >> 2;
  const int erow = q4 * 32 + lane;  // this thread's accumulator row (tensor-memory lane)
  bool ok = true;
  issue(0, 0);
  for (int it = 0; it < total; ++it) {
    const int st = it & 1, sb = it % nsb, tok_base = tile_base(it);
    cp_async_wait_all();
    if (p.use_tma && !mbar_wait(&sbar[st], static_cast<uint32_t>((it >> 1) & 1))) ok = false;
    // CTA-uniform: a wait that expired in any thread ends the loop for all.
    if (__syncthreads_or(!ok)) break;
    ph.mark(0);
    if (it + 1 < total) issue(it + 1, st ^ 1);
    // Widen this stage's 4-bit weight quants into the MMA layout, and form
    // each token's eight 32-value sums of its activation quants.
    const uint8_t* araw = sm + kOffARaw + st * 2 * kARawBytes;
    const uint8_t* meta = sm + kOffBMeta + st * kBMetaBytes;
    if (tid < NMAT * kTcRows) {
      const int m = tid / kTcRows, r = tid % kTcRows;
      const uint4* qsrc = reinterpret_cast<const uint4*>(araw + (m * kTcRows + r) * kARawRow + 16);
      uint8_t* aop = sm + kOffAOp + m * kAOpBytes;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
          const uint4 q = qsrc[2 * c + kc];
          const uint4 lo = make_uint4(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu);
          const uint4 hi = make_uint4((q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu, (q.z >> 4) & 0x0F0F0F0Fu,
                                      (q.w >> 4) & 0x0F0F0F0Fu);
          *reinterpret_cast<uint4*>(aop + (2 * c) * (kTcRows * 32) + core_off(r, kc)) = lo;
          *reinterpret_cast<uint4*>(aop + (2 * c + 1) * (kTcRows * 32) + core_off(r, kc)) = hi;
        }
      }
    }
    {
      const int t = tid >> 3, j = tid & 7;  // kTcThreads == kTcTok * 8
      const int w = reinterpret_cast<const int*>(meta + t * 48)[j];
      bsp[t * 8 + j] = lo16(w) + hi16(w);
    }
    fence_async_smem();
    __syncthreads();
    ph.mark(1);
    if (tid == 0) {
      tc_fence_after();
      const uint32_t aop0 = smem_u32(sm + kOffAOp);
      const uint32_t bop0 = smem_u32(sm + kOffBOp + st * kBOpBytes);
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int j = 0; j < kTcKBlocks; ++j)
          tc_mma(tmem + static_cast<uint32_t>((m * kTcKBlocks + j) * kTcTok),
                 smem_desc(aop0 + m * kAOpBytes + j * (kTcRows * 32)), smem_desc(bop0 + j * (kTcTok * 32)));
      tc_commit(bar);
    }
    if (!mbar_wait(bar, static_cast<uint32_t>(it & 1))) ok = false;
    if (__syncthreads_or(!ok)) break;
    tc_fence_after();
    ph.mark(2);
    // Epilogue of super-block sb.
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint4 h = *reinterpret_cast<const uint4*>(araw + (m * kTcRows + erow) * kARawRow);
      const uint32_t sca = h.y & 0x3F3F3F3Fu, mna = h.z & 0x3F3F3F3Fu;
      const uint32_t scb = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
      const uint32_t mnb = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
      int sumi[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) sumi[t] = 0;
      // kTcLdBatch sub-block accumulators per tensor-memory round trip; the
      // integer sums still run over j in order.
#pragma unroll
      for (int j0 = 0; j0 < kTcKBlocks; j0 += kTcLdBatch) {
        int v[kTcLdBatch][16];
#pragma unroll
        for (int u = 0; u < kTcLdBatch; ++u)
          tc_ld16_issue(tmem + (static_cast<uint32_t>(q4 * 32) << 16) +
                            static_cast<uint32_t>((m * kTcKBlocks + j0 + u) * kTcTok + th * 16),
                        v[u]);
        tc_wait_ld();
#pragma unroll
        for (int u = 0; u < kTcLdBatch; ++u) {
          const int j = j0 + u;
          const int s = byte_of(j < 4 ? sca : scb, j & 3);
#pragma unroll
          for (int t = 0; t < 16; ++t) sumi[t] += s * v[u][t];
        }
      }
      const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
      int mn[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mn[j] = byte_of(j < 4 ? mna : mnb, j & 3);
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const int tok = th * 16 + t;
        const int4 b0 = *reinterpret_cast<const int4*>(bsp + tok * 8);
        const int4 b1 = *reinterpret_cast<const int4*>(bsp + tok * 8 + 4);
        const float yd = *reinterpret_cast<const float*>(meta + tok * 48 + 32);
        const int summ = mn[0] * b0.x + mn[1] * b0.y + mn[2] * b0.z + mn[3] * b0.w + mn[4] * b1.x + mn[5] * b1.y +
                         mn[6] * b1.z + mn[7] * b1.w;
        tree[m][t].add(sb, __fsub_rn(__fmul_rn(__fmul_rn(d, yd), static_cast<float>(sumi[t])),
                                     __fmul_rn(__fmul_rn(dmin, yd), static_cast<float>(summ))));
      }
    }
    tc_fence_before();
    ph.mark(3);
    if (sb == nsb - 1) {
      // The tile is complete: its outputs.
      const int row = row0 + erow;
      if (row < p.rows) {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int tok = tok_base + th * 16 + t;
          if (tok >= t_cnt) break;
          const int o = p.out_idx != nullptr ? p.out_idx[t_off + tok] : tok;
          float* dst = p.out + static_cast<int64_t>(o) * p.out_stride + row;
          const float v = tree[0][t].r;
          if (p.mode == 0) {
            *dst = v;
          } else if (p.mode == 1) {
            *dst = __fadd_rn(*dst, v);
          } else if (NMAT == 2) {
            const float sl = __fdiv_rn(v, __fadd_rn(1.0f, exp_cw(-v)));
            *dst = __fmul_rn(sl, tree[NMAT - 1][t].r);
          }
        }
      }
    }
  }
  cp_async_wait_all();
  if (!ok) {
    if (lane == 0 && p.err != nullptr) atomicCAS(p.err, 0, NH_E_TIMEOUT);
    // Give the in-flight MMAs and tensor-map loads a last bounded chance to
    // finish before the tensor memory and the CTA's shared memory are released.
    (void)mbar_wait(bar, 0u);
    (void)mbar_wait(bar, 1u);
    if (p.use_tma) {
      for (int s2 = 0; s2 < 2; ++s2) {
        (void)mbar_wait(&sbar[s2], 0u);
        (void)mbar_wait(&sbar[s2], 1u);
      }
    }
  }
  ph.store();
  phase_value(6, static_cast<unsigned long long>(total));
  phase_value(7, static_cast<unsigned long long>(NMAT));
  phase_end(kPhGroupedTc, ph_idx);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kCols) : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link the driver API); null when unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// A 2-D tensor map over n_rows rows of rb bytes (Q4_K rows) read in boxes of
// one 144-byte block x kTcRows rows; rows past the end read as zero.
bool encode_q4k_rows(CUtensorMap* m, const void* base, uint64_t rb, uint64_t n_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr || n_rows == 0 || n_rows > 0x7fffffffull || rb % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return false;
  const cuuint64_t dims[2] = {rb, n_rows};
  const cuuint64_t strides[1] = {rb};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kARawRow), static_cast<cuuint32_t>(kTcRows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor-map weight loads are on unless NH_TC_TMA=0 (read once).
bool tc_tma_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = std::getenv("NH_TC_TMA");
    v = (s != nullptr && s[0] == '0') ? 0 : 1;
  }
  return v != 0;
}

// Whether the tensor-core form is enabled (NH_TC=0 turns it off; read once).
bool tc_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = std::getenv("NH_TC");
    v = (s != nullptr && s[0] == '0') ? 0 : 1;
  }
  return v != 0;
}

}  // namespace

}  // namespace nh

using namespace nh;

extern "C" int nh_batch_rowdot_tc(const NhGroupedRowDot* g, void* stream) {
  if (g == nullptr || g->w == nullptr || g->q8 == nullptr || g->out == nullptr || g->rows <= 0 || g->n_groups <= 0 ||
      g->max_tokens <= 0)
    return NH_E_ARG;
  const bool swiglu = g->mode == NH_ROWDOT_SWIGLU;
  if (g->type != NH_TYPE_Q4_K || (swiglu && (g->w2 == nullptr || g->type2 != NH_TYPE_Q4_K))) return NH_E_TYPE;
  if (g->n < QK || g->n % QK != 0 || g->n / QK > 8 || (g->n / QK & (g->n / QK - 1)) != 0) return NH_E_ARG;
  if (g->mode != NH_ROWDOT_STORE && g->mode != NH_ROWDOT_RESIDUAL && !swiglu) return NH_E_ARG;
  if (g->off == nullptr && g->n_tok <= 0) return NH_E_ARG;
  // cp.async moves 16-byte chunks: weights, rows and activation blocks must be 16-byte aligned.
  const uint64_t rb = static_cast<uint64_t>(g->n / QK) * kQ4KBytes;
  if ((reinterpret_cast<uintptr_t>(g->w) & 15) != 0 || (g->w2 != nullptr && (reinterpret_cast<uintptr_t>(g->w2) & 15)) ||
      (reinterpret_cast<uintptr_t>(g->q8) & 15) != 0 || (g->mstride & 15) != 0 || (g->mstride2 & 15) != 0)
    return NH_E_ARG;
  TcArgs p;
  memset(&p, 0, sizeof(p));
  p.w = static_cast<const uint8_t*>(g->w);
  p.w2 = static_cast<const uint8_t*>(g->w2);
  p.mstride = g->mstride;
  p.mstride2 = g->mstride2;
  p.rb = rb;
  p.K = static_cast<int>(g->n);
  p.rows = static_cast<int>(g->rows);
  p.row_tiles = (p.rows + kTcRows - 1) / kTcRows;
  p.mode = g->mode;
  p.n_tok = g->n_tok;
  p.off = g->off;
  p.cnt = g->cnt;
  p.act_idx = g->act_idx;
  p.out_idx = g->out_idx;
  p.q8 = static_cast<const uint8_t*>(g->q8);
  p.out = g->out;
  p.out_stride = g->out_stride;
  p.err = g->err;
  // The weight tiles come by tensor-map loads when every group's rows are
  // contiguous (group g's rows start g * rows * rb after the first), else by
  // per-row cp.async (e.g. slot pools with padded slots).
  {
    const uint64_t groups = static_cast<uint64_t>(g->n_groups);
    const uint64_t span = static_cast<uint64_t>(p.rows) * rb;
    const bool contiguous = groups == 1 || (g->mstride == span && (!swiglu || g->mstride2 == span));
    p.use_tma = tc_tma_enabled() && contiguous && encode_q4k_rows(&p.tmap[0], g->w, rb, groups * p.rows) &&
                (!swiglu || encode_q4k_rows(&p.tmap[1], g->w2, rb, groups * p.rows))
                    ? 1
                    : 0;
  }
  // Grouped products: a CTA walks its group's token tiles y, y + grid.y, ...;
  // two CTAs per (group, row tile) cover the usual per-expert token counts
  // without launching mostly-empty tiles.  Dense products: one tile each.
  const int tiles = (g->max_tokens + kTcTok - 1) / kTcTok;
  const dim3 grid(static_cast<unsigned>(g->n_groups * p.row_tiles),
                  static_cast<unsigned>(g->off != nullptr ? std::min(tiles, 2) : tiles));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (swiglu) {
    static SmemLimit configured;
    if (!ensure_smem(grouped_q4k_tc_kernel<2>, kTcSmemBytes, configured)) return NH_E_CUDA;
    return launch_pdl(grouped_q4k_tc_kernel<2>, grid, dim3(kTcThreads), kTcSmemBytes, st, p);
  }
  static SmemLimit configured1;
  if (!ensure_smem(grouped_q4k_tc_kernel<1>, kTcSmemBytes, configured1)) return NH_E_CUDA;
  return launch_pdl(grouped_q4k_tc_kernel<1>, grid, dim3(kTcThreads), kTcSmemBytes, st, p);
}

extern "C" int nh_tc_enabled(void) { return tc_enabled() ? 1 : 0; }

NH_PHASE_TRACE_SETTER(grouped_tc)

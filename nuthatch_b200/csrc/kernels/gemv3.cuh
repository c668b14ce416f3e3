// GEMV work split shared by the batch-1 projection kernels: weight segments
// (up to three, e.g. Q, K and V), jobs of 32/G rows each staged by the warp's
// cp.async.bulk ring, and the lane-per-super-block job loop (rowdot3.cuh).
#pragma once

#include "rowdot3.cuh"

namespace nh {

constexpr int kGemvWarps = 8;
constexpr int kGemvMaxStages = 4;
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
  int S;  // ring depth (<= kGemvMaxStages)
  const float* x;
  const float* norm_w;
  float eps;
  int do_norm;
  int quant;
  int need_wf;  // stage norm_w in shared memory
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

// The lane-per-super-block work split of a GemvArgs whose segments (all
// quantised), K and activation source are set: G = K/256 lanes per row, jobs
// of P = 32/G rows, staging buffers for the widest row (ring depth S left to
// the caller).
inline void gemv3_shape(GemvArgs& p) {
  uint64_t rb_max = 0;
  for (int s = 0; s < p.nseg; ++s) {
    p.seg[s].rb = row_bytes(p.seg[s].type, p.K);
    rb_max = rb_max > p.seg[s].rb ? rb_max : p.seg[s].rb;
  }
  p.quant = 1;
  p.need_wf = (p.do_norm != 0 && p.norm_w != nullptr) ? 1 : 0;
  p.lpr = p.K / QK;
  p.rpp = 32 / p.lpr;
  int total = 0;
  for (int s = 0; s < p.nseg; ++s) {
    p.jobs_start[s] = total;
    total += (p.seg[s].rows + p.rpp - 1) / p.rpp;
  }
  for (int s = p.nseg; s < 4; ++s) p.jobs_start[s] = total;
  p.jobs_total = total;
  p.stage_bytes = static_cast<uint32_t>((rb_max * p.rpp + 32 + 127) & ~127ull);
}

// Lane 0 stages job j (a quantised segment) into stage st of the warp's ring.
__device__ __forceinline__ void g3_issue(const GemvArgs& p, uint64_t* wbar, uint8_t* wb, int j, int st, int lane) {
  if (lane != 0) return;
  int s, row0, nrows;
  gemv_job(p, j, s, row0, nrows);
  uint32_t len, off;
  const uint8_t* src = span16(p.seg[s].w + static_cast<uint64_t>(row0) * p.seg[s].rb,
                              static_cast<size_t>(nrows) * p.seg[s].rb, &len, &off);
  mbar_expect_tx(&wbar[st], len);
  bulk_g2s(wb + static_cast<size_t>(st) * p.stage_bytes, src, len, &wbar[st]);
}

// The warp's jobs gw, gw+tw, ... (the first S already issued) of quantised
// segments without argmax: out[row] = resid[row] + (W.x)[row] (or the bare
// dot without resid).  Returns false when a stage wait expired.
template <class View>
__device__ __forceinline__ bool g3_run(const GemvArgs& p, uint64_t* wbar, uint8_t* wb, const View& act, int gw,
                                       int tw, int lane) {
  const int G = p.lpr;
  const int g = lane % G, r = lane / G;
  for (int it = 0;; ++it) {
    const int j = gw + it * tw;
    if (j >= p.jobs_total) break;
    const int st = it % p.S;
    int s, row0, nrows;
    gemv_job(p, j, s, row0, nrows);
    const GemvSeg& sg = p.seg[s];
    if (!mbar_wait(&wbar[st], (it / p.S) & 1)) return false;
    const uint32_t off =
        static_cast<uint32_t>(reinterpret_cast<uintptr_t>(sg.w + static_cast<uint64_t>(row0) * sg.rb) & 15);
    const uint8_t* rowp = wb + static_cast<size_t>(st) * p.stage_bytes + off + static_cast<size_t>(r) * sg.rb;
    float v = row_dot3v(rowp, sg.type, g, G, act);
    const int row = row0 + r;
    if (g == 0 && r < nrows) {
      if (sg.resid != nullptr) v = __fadd_rn(sg.resid[row], v);
      sg.out[row] = v;
    }
    __syncwarp();
    const int jn = gw + (it + p.S) * tw;
    if (jn < p.jobs_total) g3_issue(p, wbar, wb, jn, st, lane);
  }
  return true;
}

}  // namespace nh

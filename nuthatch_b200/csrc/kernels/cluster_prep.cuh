// Activation preparation shared by the CTAs of a thread-block cluster.
//
// Every CTA of a row-dot kernel needs the whole prepared activation (RMS
// normalised, optionally multiplied by a norm weight, Q8_K-quantised).
// Instead of each CTA loading and preparing all K values, CTA `rank` of a
// cluster of C loads and normalises the element slice [rank*K/C,
// (rank+1)*K/C), quantises the Q8_K blocks of that slice, and writes the
// results into every CTA's shared memory through distributed shared memory.
// The RMS sum of squares is formed per CTA over its slice and the C partial
// sums are added in rank order by every CTA, so all CTAs use one scale.
//
// Launched without a cluster, the cluster has one CTA and this is the local
// preparation.  Requirements checked by the launchers: K % (4*C) == 0, and
// for quantisation (K/256) % C == 0 (each rank owns whole blocks).
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace nh {

namespace cg = cooperative_groups;

// Cluster barrier halves.  Every CTA arrives once at kernel start and waits
// before its first access to another CTA's shared memory, which guarantees
// that all CTAs of the cluster are running by then.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory"); }

// Stages this CTA's slice of the RMSNorm weight (static data: callers issue it
// before griddepcontrol.wait).
__device__ inline void cluster_load_norm(ActSmem& a, const float* __restrict__ norm_w) {
  if (a.wf == nullptr || norm_w == nullptr) return;
  cg::cluster_group cl = cg::this_cluster();
  const int C = static_cast<int>(cl.num_blocks()), rank = static_cast<int>(cl.block_rank());
  const int es = a.K / C, e0 = rank * es;
  copy_to_smem(a.wf + e0, norm_w + e0, es);
}

// See the file comment.  s_part holds >= 8 doubles of shared memory, red >=
// 33.  full_f32: also give every CTA the whole normalised f32 row in a.xf.
// Ends with a cluster-wide barrier.
__device__ inline void cluster_prep_act(ActSmem& a, const float* __restrict__ src, bool has_norm_w, bool do_norm,
                                        float eps, bool quant, bool full_f32, double* red, double* s_part) {
  cg::cluster_group cl = cg::this_cluster();
  const int C = static_cast<int>(cl.num_blocks()), rank = static_cast<int>(cl.block_rank());
  const int K = a.K, es = K / C, e0 = rank * es;
  const int tid = threadIdx.x, nt = blockDim.x, warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
  copy_to_smem(a.xf + e0, src + e0, es);
  __syncthreads();
  float scale = 1.f;
  if (do_norm) {
    double s = 0.0;
    for (int i = tid; i < es; i += nt) {
      const float v = a.xf[e0 + i];
      s += static_cast<double>(__fmul_rn(v, v));
    }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid < C) {
      double t = 0.0;
      for (int w = 0; w < nw; ++w) t += red[w];
      *cl.map_shared_rank(s_part + rank, tid) = t;
    }
    cl.sync();
    double t = 0.0;
    for (int r = 0; r < C; ++r) t += s_part[r];
    const float mean = static_cast<float>(t / static_cast<double>(K));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    const bool w = has_norm_w && a.wf != nullptr;
    for (int i = tid; i < es; i += nt) {
      float v = __fmul_rn(a.xf[e0 + i], scale);
      if (w) v = __fmul_rn(v, a.wf[e0 + i]);
      a.xf[e0 + i] = v;
    }
  }
  __syncthreads();
  if (full_f32 && C > 1) {
    // The normalised slice to every other CTA (16-byte stores).
    const int n4 = es / 4;
    const float4* mine = reinterpret_cast<const float4*>(a.xf + e0);
    for (int q = tid; q < n4 * (C - 1); q += nt) {
      const int r = (rank + 1 + q / n4) % C, i = q % n4;
      *cl.map_shared_rank(reinterpret_cast<float4*>(a.xf + e0) + i, r) = mine[i];
    }
  }
  if (quant) {
    const int nbr = es / QK, b0 = e0 / QK;  // this rank's blocks
    for (int bb = warp; bb < nbr; bb += nw) {
      const int b = b0 + bb;
      const float4 v0 = *reinterpret_cast<const float4*>(a.xf + b * QK + lane * 8);
      const float4 v1 = *reinterpret_cast<const float4*>(a.xf + b * QK + lane * 8 + 4);
      const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      quantize_block_warp(v, b, a, lane);
    }
    if (C > 1) {
      __syncthreads();
      // Per block: 256 quant bytes (16 x 16 B), 16 sums (2 x 16 B), the scale.
      const int per = 19;
      for (int q = tid; q < nbr * per * (C - 1); q += nt) {
        const int r = (rank + 1 + q / (nbr * per)) % C;
        const int rem = q % (nbr * per), b = b0 + rem / per, part = rem % per;
        if (part < 16) {
          const uint4* s4 = reinterpret_cast<const uint4*>(a.qs + b * QK) + part;
          *cl.map_shared_rank(const_cast<uint4*>(s4), r) = *s4;
        } else if (part < 18) {
          const uint4* s4 = reinterpret_cast<const uint4*>(a.bsums + b * 16) + (part - 16);
          *cl.map_shared_rank(const_cast<uint4*>(s4), r) = *s4;
        } else {
          *cl.map_shared_rank(a.d + b, r) = a.d[b];
        }
      }
    }
  }
  cl.sync();
}

}  // namespace nh

// Embedding lookup for the decode cursor, and the standalone Q8_K
// quantisation / K-quant dequantisation entry points the parity tests use.
#include "common.cuh"
#include "launch.cuh"

namespace nh {

// ggml dequantize_row_* element formulas (both products rounded before the
// subtraction, as the f32 reference does).
__device__ __forceinline__ float dequant_elem(const uint8_t* row, int type, int64_t i) {
  if (type == NH_TYPE_F32) return reinterpret_cast<const float*>(row)[i];
  const int64_t b = i / QK;
  const int e = static_cast<int>(i % QK);
  if (type == NH_TYPE_Q4_K) {
    const uint8_t* blk = row + b * kQ4KBytes;
    const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
    const float dmin = half_bits_to_float(blk[2] | (blk[3] << 8));
    const int j = e / 32, c = j / 2;
    int sc, m;
    q4k_scale_min(blk + 4, j, sc, m);
    const uint8_t byte = blk[16 + 32 * c + (e % 32)];
    const int q = (j & 1) ? (byte >> 4) : (byte & 15);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                     __fmul_rn(dmin, static_cast<float>(m)));
  }
  const uint8_t* blk = row + b * kQ6KBytes;
  const float d = half_bits_to_float(blk[208] | (blk[209] << 8));
  const int h = e / 128, ee = e % 128;
  const int lo = ee < 64 ? (blk[64 * h + ee] & 15) : (blk[64 * h + ee - 64] >> 4);
  const int hi = (blk[128 + 32 * h + ee % 32] >> (2 * (ee / 32))) & 3;
  const int q = (lo | (hi << 4)) - 32;
  const int8_t sc = static_cast<int8_t>(blk[192 + e / 16]);
  return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
}

// One warp: the k selected ids to mapped host memory, then (after a
// system-scope fence) the sequence number the host waits for.
__global__ void publish_kernel(const int32_t* sel, int k, int32_t* host_sel, unsigned* host_seq, unsigned seq) {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int lane = threadIdx.x;
  if (lane < k) host_sel[lane] = sel[lane];
  __threadfence_system();
  __syncwarp();
  if (lane == 0) *reinterpret_cast<volatile unsigned*>(host_seq) = seq;
}

__global__ void embed_kernel(const NhDecodeState* state, const int32_t* prompt, const uint8_t* table,
                             int type, int64_t n_embd, int64_t n_vocab, uint64_t rb, float* h) {
  phase_end(kPhEmbed, phase_begin());
  __shared__ int s_tok;
  // The fed-back id comes from the preceding argmax.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (threadIdx.x == 0) {
    const int pos = state->pos;
    int tok = pos < state->n_prompt ? prompt[pos] : state->token;
    if (tok < 0 || tok >= n_vocab) {
      atomicCAS(const_cast<int32_t*>(&state->error), 0, NH_E_ARG);
      tok = 0;
    }
    s_tok = tok;
  }
  __syncthreads();
  // Stage the row with 16-byte loads from its 16-byte-rounded start (weight
  // regions carry tail padding), then dequantise from shared memory.
  extern __shared__ __align__(16) uint8_t row_s[];
  const uintptr_t a = reinterpret_cast<uintptr_t>(table + static_cast<uint64_t>(s_tok) * rb);
  const uintptr_t al = a & ~static_cast<uintptr_t>(15);
  const int off = static_cast<int>(a - al);
  const int n16 = static_cast<int>((off + rb + 15) >> 4);
  const uint4* g = reinterpret_cast<const uint4*>(al);
  for (int k = threadIdx.x; k < n16; k += blockDim.x) reinterpret_cast<uint4*>(row_s)[k] = g[k];
  __syncthreads();
  const uint8_t* row = row_s + off;
  for (int64_t i = threadIdx.x; i < n_embd; i += blockDim.x) h[i] = dequant_elem(row, type, i);
}

__global__ void dequant_kernel(const uint8_t* w, int type, int64_t n, int64_t rows, uint64_t rb, float* y) {
  const int64_t total = n * rows;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / n, i = idx % n;
    y[idx] = dequant_elem(w + r * rb, type, i);
  }
}

// One CTA per 256-value block: prep_act's quantiser over a one-block row.
__global__ void quantize_kernel(const float* x, int64_t n, uint8_t* out) {
  __shared__ __align__(16) uint8_t smem[4096];
  __shared__ double red[48];
  ActSmem a = carve_act(smem, QK, true);
  prep_act(a, x + static_cast<int64_t>(blockIdx.x) * QK, false, false, 0.f, true, red);
  uint8_t* blk = out + static_cast<int64_t>(blockIdx.x) * 292;
  if (threadIdx.x == 0) *reinterpret_cast<float*>(blk) = a.d[0];
  for (int i = threadIdx.x; i < QK; i += blockDim.x) blk[4 + i] = static_cast<uint8_t>(a.qs[q8_off(0, i)]);
  for (int i = threadIdx.x; i < 16; i += blockDim.x) {
    const int16_t v = a.bsums[i];
    blk[260 + 2 * i] = static_cast<uint8_t>(v & 0xFF);
    blk[261 + 2 * i] = static_cast<uint8_t>((v >> 8) & 0xFF);
  }
}

__global__ void exp_cw_kernel(const float* x, int64_t n, float* y) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = exp_cw(x[i]);
}

}  // namespace nh

using namespace nh;

extern "C" int nh_exp_cw(const float* x, int64_t n, float* y, void* stream) {
  if (x == nullptr || y == nullptr || n <= 0) return NH_E_ARG;
  const int grid = static_cast<int>(std::min<int64_t>(1024, (n + 255) / 256));
  exp_cw_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, y);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

extern "C" int nh_publish_selection(const int32_t* sel, int k, int32_t* host_sel, uint32_t* host_seq, uint32_t seq,
                                    void* stream) {
  if (sel == nullptr || host_sel == nullptr || host_seq == nullptr || k <= 0 || k > 32) return NH_E_ARG;
  return launch_pdl(publish_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), sel, k, host_sel,
                    static_cast<unsigned*>(host_seq), static_cast<unsigned>(seq));
}

extern "C" int nh_embed_step(const NhDecodeState* state, const int32_t* prompt_ids, const void* table,
                             int32_t type, int64_t n_embd, int64_t n_vocab, float* h_out, void* stream) {
  if (state == nullptr || prompt_ids == nullptr || table == nullptr || h_out == nullptr) return NH_E_ARG;
  if (type != NH_TYPE_F32 && type != NH_TYPE_Q4_K && type != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (type != NH_TYPE_F32 && n_embd % QK != 0) return NH_E_ARG;
  const size_t smem = row_bytes(type, n_embd) + 32;
  static SmemLimit configured;
  if (smem > 220 * 1024 || !ensure_smem(embed_kernel, smem, configured)) return NH_E_ARG;
  return launch_pdl(embed_kernel, dim3(1), dim3(256), smem, static_cast<cudaStream_t>(stream), state, prompt_ids,
                    static_cast<const uint8_t*>(table), static_cast<int>(type), n_embd, n_vocab,
                    static_cast<uint64_t>(row_bytes(type, n_embd)), h_out);
}

extern "C" int nh_dequantize(const void* w, int32_t type, int64_t n, int64_t rows, float* y, void* stream) {
  if (w == nullptr || y == nullptr || n <= 0 || rows <= 0) return NH_E_ARG;
  if (type != NH_TYPE_F32 && type != NH_TYPE_Q4_K && type != NH_TYPE_Q6_K) return NH_E_TYPE;
  if (type != NH_TYPE_F32 && n % QK != 0) return NH_E_ARG;
  const int64_t total = n * rows;
  int grid = static_cast<int>((total + 255) / 256);
  if (grid > 4096) grid = 4096;
  dequant_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w), type, n, rows, row_bytes(type, n), y);
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

extern "C" int nh_quantize_q8k(const float* x, int64_t n, void* out, void* stream) {
  if (x == nullptr || out == nullptr || n <= 0 || n % QK != 0) return NH_E_ARG;
  quantize_kernel<<<static_cast<int>(n / QK), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, n, static_cast<uint8_t*>(out));
  return cudaGetLastError() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

NH_PHASE_TRACE_SETTER(misc)

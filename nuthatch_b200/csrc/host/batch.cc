// Batched greedy decode: GreedyGenerateCachedBatch (no reference
// counterpart; the batched form of generate.cc:55-106 for serving many
// sequences at once).  B sequences of equal prompt length advance one
// position per step in lockstep; every step is one sequence of kernel
// launches (nh_batch_* in nh_kernels.h), captured once as a CUDA graph and
// replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <unordered_map>

#include "engine.h"
#include "nccl_api.h"
#include "nuthatch/expert_parallel.h"
#include "nuthatch/expert_slot_cache.h"
#include "nuthatch/streaming_forward.h"
#include "nuthatch/streaming_model.h"
#include "wave_plan.h"
#include "workspace.h"
#include "nuthatch/generate.h"
#include "nuthatch/gguf_file.h"

namespace nuthatch {

namespace {

// Device buffers of one batched generation.
class BatchBuffers {
 public:
  ~BatchBuffers() {
    for (void* p : owned_) cudaFree(p);
    for (void* p : host_owned_) cudaFreeHost(p);
    if (graph_ != nullptr) cudaGraphExecDestroy(graph_);
    if (event_ != nullptr) cudaEventDestroy(event_);
    if (stream_ != nullptr) cudaStreamDestroy(stream_);
  }
  template <typename T>
  T* Alloc(size_t count) {
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
      ok_ = false;
      return nullptr;
    }
    owned_.push_back(p);
    return static_cast<T*>(p);
  }
  // Pinned host memory (freed with the buffers).
  template <typename T>
  T* HostAlloc(size_t count) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, std::max<size_t>(count, 1) * sizeof(T), cudaHostAllocDefault) != cudaSuccess) {
      ok_ = false;
      return nullptr;
    }
    host_owned_.push_back(p);
    return static_cast<T*>(p);
  }
  bool ok_ = true;
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;
  cudaEvent_t event_ = nullptr;

 private:
  std::vector<void*> owned_;
  std::vector<void*> host_owned_;
};

// All-gather of every rank's Q8_K activation rows and top-k selections
// (rank r's block at r * the block size).
int ExchangeTokens(const ExpertGroup& ep, const uint8_t* q8, size_t q8_bytes, uint8_t* q8_all, const int32_t* sel,
                   size_t n_sel, int32_t* sel_all, cudaStream_t s) {
  const NcclApi& n = Nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ep.comm());
  if (n.GroupStart() != ncclSuccess) return NH_E_CUDA;
  const bool ok = n.AllGather(q8, q8_all, q8_bytes, ncclUint8, comm, s) == ncclSuccess &&
                  n.AllGather(sel, sel_all, n_sel, ncclInt32, comm, s) == ncclSuccess;
  return n.GroupEnd() == ncclSuccess && ok ? NH_OK : NH_E_CUDA;
}

// All-to-all of the pick rows: block r of y (rank r's tokens' picks, rows
// (token, slot) in order; only picks of experts this rank owns are
// meaningful) goes to rank r, and block q of y_recv arrives from rank q.
int ReturnPicks(const ExpertGroup& ep, const float* y, size_t block, float* y_recv, cudaStream_t s) {
  const NcclApi& n = Nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ep.comm());
  if (n.GroupStart() != ncclSuccess) return NH_E_CUDA;
  bool ok = true;
  for (int r = 0; r < ep.world() && ok; ++r) {
    ok = n.Send(y + r * block, block, ncclFloat32, r, comm, s) == ncclSuccess &&
         n.Recv(y_recv + r * block, block, ncclFloat32, r, comm, s) == ncclSuccess;
  }
  return n.GroupEnd() == ncclSuccess && ok ? NH_OK : NH_E_CUDA;
}

#define NH_B_TRY(x)             \
  do {                          \
    const int rc_ = (x);        \
    if (rc_ != NH_OK) return rc_; \
  } while (0)

// The chunked prompt prefill of the batched decode is on unless
// NH_BATCH_PREFILL=0 (read at every call).
bool BatchPrefillEnabled() {
  const char* e = std::getenv("NH_BATCH_PREFILL");
  return !(e != nullptr && e[0] == '0');
}

// Rows of one prefill chunk (sequences x positions), at most.
constexpr int kBatchPrefillRows = 512;

// Prompts of equal, non-zero length with ids inside the vocabulary.
int CheckPrompts(const std::vector<std::vector<int32_t>>& prompts, const OlmoeConfig& c) {
  const size_t P = prompts[0].size();
  for (const auto& p : prompts) {
    if (p.size() != P || P == 0) return NH_E_ARG;
    for (int32_t t : p)
      if (t < 0 || static_cast<uint32_t>(t) >= c.n_vocab) return NH_E_ARG;
  }
  return NH_OK;
}

// Experts streamed through per-layer slot pools (the batched streaming form):
// the caches, the stream their fills run on, the experts this GPU serves
// (all of them, or its expert-parallel shard) and the wave statistics.
struct StreamedExperts {
  std::vector<ExpertSlotCache*> caches;
  cudaStream_t copy_stream = nullptr;
  ExpertShard shard;
  int64_t waves = 0;      // out: slot-pool waves over all layers and steps
  double host_ms = 0;     // out: host time spent in slot decisions and waits
};

int StreamedMoe(StreamedExperts& se, int l, const OlmoeConfig& c, int B, const int32_t* sel, int32_t* sel_host,
                int32_t* plan_host, int32_t* off, int32_t* cnt, int32_t* act_idx, int32_t* out_idx,
                const uint8_t* q8, float* ff, uint8_t* q8ff, float* y, cudaEvent_t compute_done, cudaStream_t s);

// The batched decode shared by the resident (and expert-parallel) form and the
// streaming form: `se` null means the experts are resident in `m` (offset by
// e_skip experts), else they are streamed through se's slot pools.
std::vector<std::vector<int32_t>> RunBatch(const ModelView& m, const OlmoeConfig& c,
                                           const std::vector<std::vector<int32_t>>& prompts, int n_predict,
                                           bool norm_topk, BatchOptions& o, ExpertShard shard, uint64_t e_skip,
                                           StreamedExperts* se) {
  std::vector<std::vector<int32_t>> out;
  const int B = static_cast<int>(prompts.size());
  const int P = static_cast<int>(prompts[0].size());
  const int64_t d = c.n_embd, hd = c.head_dim(), dkv = static_cast<int64_t>(c.n_head_kv) * hd, F = c.n_ff,
                E = c.n_expert, K = c.n_expert_used, V = c.n_vocab, L = c.n_layers;
  const ExpertGroup* ep = o.ep;
  const int W = ep != nullptr ? ep->world() : 1;
  const int max_seq = P + n_predict;
  // Chunked prompt prefill (the reference forwards the whole prompt in its
  // first step, generate.cc:63-91): positions 0..P-2 of every local sequence,
  // C positions at a time as B*C rows, through the batched kernels; the last
  // prompt position is the first decode step, which forms the logits.  Every
  // rank of an expert-parallel group has the same B and P, so the same C and
  // the same collectives.  In the streaming form each chunk's experts stream
  // through the slot pools in waves, as in a decode step.
  const bool prefill = P > 1 && BatchPrefillEnabled() && Engine::PrefillSupported(m, se == nullptr);
  const int C = prefill ? std::max(1, std::min(P - 1, kBatchPrefillRows / B)) : 1;
  const int R = prefill ? std::max(B, B * C) : B;  // rows of the largest pass
  const int RK = R * static_cast<int>(K);
  const int RW = R * W, RKW = RK * W;  // rows of every rank's tokens / picks
  BatchBuffers bb;
  NhDecodeState* state = bb.Alloc<NhDecodeState>(1);
  int32_t* prm = bb.Alloc<int32_t>(static_cast<size_t>(B) * P);
  int32_t* fed = bb.Alloc<int32_t>(B);
  int32_t* outs = bb.Alloc<int32_t>(static_cast<size_t>(B) * n_predict);
  float* h = bb.Alloc<float>(static_cast<size_t>(R) * d);
  float* q = bb.Alloc<float>(static_cast<size_t>(R) * d);
  float* kk = bb.Alloc<float>(static_cast<size_t>(R) * dkv);
  float* v = bb.Alloc<float>(static_cast<size_t>(R) * dkv);
  float* qr = bb.Alloc<float>(static_cast<size_t>(R) * d);
  float* att = bb.Alloc<float>(static_cast<size_t>(R) * d);
  float* xn = bb.Alloc<float>(static_cast<size_t>(R) * d);
  const int64_t q8_row = nh_batch_q8_bytes(1, d);
  uint8_t* q8 = bb.Alloc<uint8_t>(q8_row * R);
  int32_t* sel = bb.Alloc<int32_t>(RK);
  float* wts = bb.Alloc<float>(RK);
  int32_t* off = bb.Alloc<int32_t>(E);
  int32_t* cnt = bb.Alloc<int32_t>(E);
  int32_t* act_idx = bb.Alloc<int32_t>(RKW);
  int32_t* out_idx = bb.Alloc<int32_t>(RKW);
  float* ff = bb.Alloc<float>(static_cast<size_t>(RKW) * F);
  uint8_t* q8ff = bb.Alloc<uint8_t>(nh_batch_q8_bytes(RKW, F));
  float* y = bb.Alloc<float>(static_cast<size_t>(RKW) * d);
  // Expert-parallel exchange buffers: every rank's activation rows and
  // selections (all-gathered), and the pick rows returned by each rank.
  uint8_t* q8_all = W > 1 ? bb.Alloc<uint8_t>(q8_row * RW) : q8;
  int32_t* sel_all = W > 1 ? bb.Alloc<int32_t>(RKW) : sel;
  float* y_recv = W > 1 ? bb.Alloc<float>(static_cast<size_t>(RKW) * d) : y;
  // Streaming: the selections read back per layer and the per-wave expert
  // lists (up to one wave per expert), in pinned host memory.
  int32_t* sel_host = nullptr;
  int32_t* plan_host = nullptr;
  if (se != nullptr) {
    sel_host = bb.HostAlloc<int32_t>(RKW);
    plan_host = bb.HostAlloc<int32_t>(static_cast<size_t>(E) * (2 * E + 2 * RKW));
    if (cudaEventCreateWithFlags(&bb.event_, cudaEventDisableTiming) != cudaSuccess) bb.ok_ = false;
    o.use_graph = false;  // the host decides every layer's slots
  }
  float* logits = bb.Alloc<float>(static_cast<size_t>(B) * V);
  float* rope = bb.Alloc<float>(static_cast<size_t>(max_seq) * hd);
  const int64_t attn_bytes = nh_batch_attention_scratch_bytes(B, c.n_head, static_cast<int>(hd), max_seq);
  uint8_t* attn_scratch = bb.Alloc<uint8_t>(attn_bytes);
  unsigned* ticket = bb.Alloc<unsigned>(16);
  float* kv = bb.Alloc<float>(static_cast<size_t>(2 * L) * B * max_seq * dkv);
  if (!bb.ok_) {
    o.status = NH_E_NOMEM;
    return out;
  }
  // Set-up on the legacy stream, finished before the decode stream starts.
  std::vector<int32_t> flat(static_cast<size_t>(B) * P);
  for (int b = 0; b < B; ++b) std::memcpy(&flat[static_cast<size_t>(b) * P], prompts[b].data(), P * 4);
  std::vector<float> cs(static_cast<size_t>(max_seq) * hd);
  nh_rope_table(c.rope_freq_base, static_cast<int>(hd), max_seq, cs.data());
  NhDecodeState st0;
  std::memset(&st0, 0, sizeof(st0));
  st0.n_prompt = P;
  st0.n_predict = n_predict;
  st0.pos = prefill ? P - 1 : 0;  // the decode steps start after the prefilled positions
  bool setup = cudaMemcpy(prm, flat.data(), flat.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemcpy(rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemcpy(state, &st0, sizeof(st0), cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemset(attn_scratch, 0, attn_bytes) == cudaSuccess && cudaMemset(ticket, 0, 64) == cudaSuccess &&
               cudaMemset(fed, 0, B * 4) == cudaSuccess &&
               cudaMemset(ff, 0, static_cast<size_t>(RKW) * F * 4) == cudaSuccess &&
               cudaMemset(y, 0, static_cast<size_t>(RKW) * d * 4) == cudaSuccess &&
               cudaMemset(y_recv, 0, static_cast<size_t>(RKW) * d * 4) == cudaSuccess &&
               cudaDeviceSynchronize() == cudaSuccess &&
               cudaStreamCreateWithFlags(&bb.stream_, cudaStreamNonBlocking) == cudaSuccess;
  if (!setup) {
    o.status = NH_E_CUDA;
    return out;
  }
  cudaStream_t s = bb.stream_;
  const float eps = c.rms_eps;
  const float kq_scale = 1.0f / std::sqrt(static_cast<float>(hd));

  // Product of one weight with nt activation rows.
  auto dense = [&](const void* w, int32_t type, int64_t rows, int64_t n, const void* act, float* o_, int64_t stride,
                   int mode, int nt) {
    NhGroupedRowDot g;
    std::memset(&g, 0, sizeof(g));
    g.w = w;
    g.type = type;
    g.type2 = type;
    g.n = n;
    g.rows = rows;
    g.n_groups = 1;
    g.n_tok = nt;
    g.max_tokens = nt;
    g.q8 = act;
    g.out = o_;
    g.out_stride = stride;
    g.mode = mode;
    return nh_batch_rowdot(&g, s);
  };
  // The MoE block of layer l over the first r rows of h (moe.cc:7-63).
  auto moe = [&](int l, const LayerView& Lv, int r) -> int {
    const int rk = r * static_cast<int>(K);
    NH_B_TRY(nh_batch_prep(h, d, r, Lv.ffn_norm, eps, 1, d, q8, xn, s));
    NH_B_TRY(nh_batch_router(xn, Lv.router, r, d, static_cast<int>(E), static_cast<int>(K), norm_topk ? 1 : 0, sel,
                             wts, s));
    if (W > 1) NH_B_TRY(ExchangeTokens(*ep, q8, q8_row * r, q8_all, sel, rk, sel_all, s));
    if (se != nullptr) {
      // The served experts stream through this GPU's pools in waves; the
      // pick rows then take the same return and combine as the resident form.
      NH_B_TRY(StreamedMoe(*se, l, c, r * W, sel_all, sel_host, plan_host, off, cnt, act_idx, out_idx, q8_all, ff,
                           q8ff, y, bb.event_, s));
      if (W > 1) {
        NH_B_TRY(ReturnPicks(*ep, y, static_cast<size_t>(rk) * d, y_recv, s));
        return nh_ep_combine(y_recv, static_cast<int64_t>(rk) * d, W, sel, wts, r, static_cast<int>(K), d,
                             static_cast<int>(shard.count), h, s);
      }
      return nh_batch_combine(y, wts, r, static_cast<int>(K), d, h, s);
    }
    // The owned experts over every rank's rows: row j of the gathered rows
    // is rank j / r's row j % r.
    NH_B_TRY(nh_batch_moe_plan_range(sel_all, r * W, static_cast<int>(K), static_cast<int>(shard.first),
                                     static_cast<int>(shard.count), off, cnt, act_idx, out_idx, s));
    NhGroupedRowDot g;
    std::memset(&g, 0, sizeof(g));
    g.w = static_cast<const uint8_t*>(Lv.gate) + e_skip * Lv.gate_nb2;
    g.w2 = static_cast<const uint8_t*>(Lv.up) + e_skip * Lv.up_nb2;
    g.mstride = Lv.gate_nb2;
    g.mstride2 = Lv.up_nb2;
    g.type = Lv.tg;
    g.type2 = Lv.tu;
    g.n = d;
    g.rows = F;
    g.n_groups = static_cast<int32_t>(shard.count);
    g.off = off;
    g.cnt = cnt;
    g.act_idx = act_idx;
    g.out_idx = out_idx;
    g.max_tokens = r * W;
    g.q8 = q8_all;
    g.out = ff;
    g.out_stride = F;
    g.mode = NH_ROWDOT_SWIGLU;
    NH_B_TRY(nh_batch_rowdot(&g, s));
    NH_B_TRY(nh_batch_prep(ff, F, static_cast<int64_t>(rk) * W, nullptr, eps, 0, F, q8ff, nullptr, s));
    std::memset(&g, 0, sizeof(g));
    g.w = static_cast<const uint8_t*>(Lv.down) + e_skip * Lv.down_nb2;
    g.mstride = Lv.down_nb2;
    g.type = Lv.td;
    g.type2 = Lv.td;
    g.n = F;
    g.rows = d;
    g.n_groups = static_cast<int32_t>(shard.count);
    g.off = off;
    g.cnt = cnt;
    g.act_idx = out_idx;  // the ff row of pair j is its (row, slot) index
    g.out_idx = out_idx;
    g.max_tokens = r * W;
    g.q8 = q8ff;
    g.out = y;
    g.out_stride = d;
    g.mode = NH_ROWDOT_STORE;
    NH_B_TRY(nh_batch_rowdot(&g, s));
    if (W > 1) {
      // Rows of rank q's picks go back to rank q; the combine takes each
      // pick's row from the block of the rank that owns its expert.
      NH_B_TRY(ReturnPicks(*ep, y, static_cast<size_t>(rk) * d, y_recv, s));
      return nh_ep_combine(y_recv, static_cast<int64_t>(rk) * d, W, sel, wts, r, static_cast<int>(K), d,
                           static_cast<int>(shard.count), h, s);
    }
    return nh_batch_combine(y, wts, r, static_cast<int>(K), d, h, s);
  };
  // Prompt positions p0..p0+cc-1 of every local sequence as B*cc rows (row
  // b*cc + i is sequence b's position p0 + i): QK-norm, RoPE, the K/V append
  // and causal attention into each sequence's own cache, everything else over
  // all rows at once; no logits are formed for these positions.
  auto prefill_chunk = [&](int p0, int cc) -> int {
    const int r = B * cc;
    NH_B_TRY(nh_prefill_embed_seqs(prm + p0, P, B, cc, m.embd, m.te, d, V, h, &state->error, s));
    for (int l = 0; l < static_cast<int>(L); ++l) {
      const LayerView& Lv = m.layers[l];
      float* kc = kv + static_cast<size_t>(2 * l) * B * max_seq * dkv;
      float* vc = kv + static_cast<size_t>(2 * l + 1) * B * max_seq * dkv;
      NH_B_TRY(nh_batch_prep(h, d, r, Lv.attn_norm, eps, 1, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wq, Lv.tq, d, d, q8, q, d, NH_ROWDOT_STORE, r));
      NH_B_TRY(dense(Lv.wk, Lv.tk, dkv, d, q8, kk, dkv, NH_ROWDOT_STORE, r));
      NH_B_TRY(dense(Lv.wv, Lv.tv, dkv, d, q8, v, dkv, NH_ROWDOT_STORE, r));
      NH_B_TRY(nh_prefill_qk_seqs(q, kk, v, Lv.q_norm, Lv.k_norm, eps, B, cc, p0, c.n_head, c.n_head_kv,
                                  static_cast<int>(hd), rope, kc, vc, max_seq, qr, s));
      NH_B_TRY(nh_prefill_attention_seqs(qr, B, cc, p0, c.n_head, c.n_head_kv, static_cast<int>(hd), kq_scale, kc, vc,
                                         max_seq, att, s));
      NH_B_TRY(nh_batch_prep(att, d, r, nullptr, eps, 0, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wo, Lv.to, d, d, q8, h, d, NH_ROWDOT_RESIDUAL, r));
      NH_B_TRY(moe(l, Lv, r));
    }
    return NH_OK;
  };
  auto step = [&]() -> int {
    NH_B_TRY(nh_batch_embed(state, prm, P, fed, B, m.embd, m.te, d, V, h, s));
    for (int l = 0; l < static_cast<int>(L); ++l) {
      const LayerView& Lv = m.layers[l];
      float* kc = kv + static_cast<size_t>(2 * l) * B * max_seq * dkv;
      float* vc = kv + static_cast<size_t>(2 * l + 1) * B * max_seq * dkv;
      NH_B_TRY(nh_batch_prep(h, d, B, Lv.attn_norm, eps, 1, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wq, Lv.tq, d, d, q8, q, d, NH_ROWDOT_STORE, B));
      NH_B_TRY(dense(Lv.wk, Lv.tk, dkv, d, q8, kk, dkv, NH_ROWDOT_STORE, B));
      NH_B_TRY(dense(Lv.wv, Lv.tv, dkv, d, q8, v, dkv, NH_ROWDOT_STORE, B));
      NH_B_TRY(nh_batch_qk(state, q, kk, v, Lv.q_norm, Lv.k_norm, eps, B, c.n_head, c.n_head_kv,
                           static_cast<int>(hd), rope, kc, vc, max_seq, qr, s));
      NH_B_TRY(nh_batch_attention(state, qr, B, c.n_head, c.n_head_kv, static_cast<int>(hd), kq_scale, kc, vc,
                                  max_seq, attn_scratch, att, s));
      NH_B_TRY(nh_batch_prep(att, d, B, nullptr, eps, 0, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wo, Lv.to, d, d, q8, h, d, NH_ROWDOT_RESIDUAL, B));
      NH_B_TRY(moe(l, Lv, B));
    }
    NH_B_TRY(nh_batch_prep(h, d, B, m.out_norm, eps, 1, d, q8, nullptr, s));
    NH_B_TRY(dense(m.out, m.tout, V, d, q8, logits, V, NH_ROWDOT_STORE, B));
    return nh_batch_argmax(state, logits, B, V, fed, outs, n_predict, ticket, s);
  };

  const int steps = P + n_predict - 1;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEventCreate(&ev0);
  cudaEventCreate(&ev1);
  int rc = NH_OK;
  cudaEvent_t ev_pre = nullptr;
  if (prefill) {
    cudaEventCreate(&ev_pre);
    cudaEventRecord(ev_pre, s);
    for (int p0 = 0; p0 < P - 1 && rc == NH_OK; p0 += C) rc = prefill_chunk(p0, std::min(C, P - 1 - p0));
  }
  const int t_start = prefill ? P - 1 : 0;
  for (int t = t_start; t < steps && rc == NH_OK; ++t) {
    if (t == P - 1) cudaEventRecord(ev0, s);  // decode: from the last prompt position on
    if (t == t_start || !o.use_graph) {
      // The first step runs eagerly: it configures the kernels' shared-memory
      // limits outside of stream capture.
      rc = step();
      if (rc == NH_OK && o.use_graph && cudaStreamSynchronize(s) == cudaSuccess) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
          rc = NH_E_CUDA;
          break;
        }
        const int rc2 = step();
        if (cudaStreamEndCapture(s, &g) != cudaSuccess || rc2 != NH_OK) rc = rc2 != NH_OK ? rc2 : NH_E_CUDA;
        if (rc == NH_OK && cudaGraphInstantiate(&bb.graph_, g, 0) != cudaSuccess) rc = NH_E_CUDA;
        if (g != nullptr) cudaGraphDestroy(g);
      }
      continue;
    }
    if (cudaGraphLaunch(bb.graph_, s) != cudaSuccess) rc = NH_E_CUDA;
  }
  cudaEventRecord(ev1, s);
  if (cudaStreamSynchronize(s) != cudaSuccess && rc == NH_OK) rc = NH_E_CUDA;
  float ms = 0.f;
  if (rc == NH_OK && cudaEventElapsedTime(&ms, ev0, ev1) == cudaSuccess) o.decode_ms = ms;
  o.prefill_ms = 0;
  if (ev_pre != nullptr) {
    if (rc == NH_OK && cudaEventElapsedTime(&ms, ev_pre, ev0) == cudaSuccess) o.prefill_ms = ms;
    cudaEventDestroy(ev_pre);
  }
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  NhDecodeState st;
  if (rc == NH_OK && cudaMemcpy(&st, state, sizeof(st), cudaMemcpyDeviceToHost) == cudaSuccess && st.error != 0)
    rc = st.error;
  if (rc != NH_OK) {
    o.status = rc;
    return out;
  }
  std::vector<int32_t> ids(static_cast<size_t>(B) * n_predict);
  if (cudaMemcpy(ids.data(), outs, ids.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
    o.status = NH_E_CUDA;
    return out;
  }
  out.resize(B);
  for (int b = 0; b < B; ++b) out[b].assign(ids.begin() + static_cast<size_t>(b) * n_predict,
                                            ids.begin() + static_cast<size_t>(b + 1) * n_predict);
  return out;
}

// The expert products of one MoE layer in the batched streaming form, over
// B token rows (every rank's rows under expert parallelism).  The selections
// are read back and the distinct unpinned experts this GPU serves are split,
// in order of first selection, into waves of at most lru_slots (pinned
// experts, always resident, join the first wave): each wave's experts are
// made resident with one Ensure (which then never evicts an expert of the same
// wave), the grouped gate/up and down products run over the slot pool for
// that wave's (token, pick) pairs, and the next wave's fills wait for those
// products.  After the last wave row j of y holds pick j's expert output for
// every pick of a served expert; the caller's combine adds them in top-k
// order, so each token's arithmetic equals the resident batch's.
int StreamedMoe(StreamedExperts& se, int l, const OlmoeConfig& c, int B, const int32_t* sel, int32_t* sel_host,
                int32_t* plan_host, int32_t* off, int32_t* cnt, int32_t* act_idx, int32_t* out_idx,
                const uint8_t* q8, float* ff, uint8_t* q8ff, float* y, cudaEvent_t compute_done, cudaStream_t s) {
  ExpertSlotCache& cache = *se.caches[l];
  const int K = static_cast<int>(c.n_expert_used), E = static_cast<int>(c.n_expert), BK = B * K;
  const int64_t d = c.n_embd, F = c.n_ff;
  const int e_lo = static_cast<int>(se.shard.first), e_hi = e_lo + static_cast<int>(se.shard.count);
  const auto t0 = std::chrono::steady_clock::now();
  if (cudaMemcpyAsync(sel_host, sel, static_cast<size_t>(BK) * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return NH_E_CUDA;
  std::vector<char> pinned(E, 0);
  for (int e = 0; e < E; ++e) pinned[e] = cache.is_pinned(e) ? 1 : 0;
  std::vector<std::vector<int>> waves;
  std::vector<int> wave_of;
  const int n_waves = PlanWaves(sel_host, BK, E, e_lo, e_hi, cache.lru_slots(), pinned, &waves, &wave_of);
  if (n_waves < 0) return n_waves;
  const int slots = static_cast<int>(cache.gate_slots()->ne[2]);
  if (slots > E) return NH_E_CAPACITY;
  const size_t plan_stride = static_cast<size_t>(2 * E + 2 * BK);
  std::vector<int> slot_of(E, -1);
  for (int w = 0; w < n_waves; ++w) {
    if (w > 0) {
      // The previous wave's products still read slots this wave may refill.
      if (cudaEventRecord(compute_done, s) != cudaSuccess ||
          cudaStreamWaitEvent(se.copy_stream, compute_done, 0) != cudaSuccess)
        return NH_E_CUDA;
    }
    const std::unordered_map<int, int> resident = cache.Ensure(waves[w]);
    if (!cache.ok()) return NH_E_IO;
    for (const auto& kv : resident) slot_of[kv.first] = kv.second;
    // This wave's pairs grouped by slot, (token, pick) order within a slot.
    int32_t* hoff = plan_host + w * plan_stride;
    int32_t* hcnt = hoff + E;
    int32_t* hact = hcnt + E;
    int32_t* hout = hact + BK;
    const int n = GroupWavePairs(sel_host, BK, K, wave_of, w, slot_of, slots, hoff, hcnt, hact, hout);
    if (n < 0) return n;
    if (cudaMemcpyAsync(off, hoff, static_cast<size_t>(slots) * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(cnt, hcnt, static_cast<size_t>(slots) * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(act_idx, hact, static_cast<size_t>(std::max(n, 1)) * 4, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaMemcpyAsync(out_idx, hout, static_cast<size_t>(std::max(n, 1)) * 4, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(cache.fills_done_event()), 0) != cudaSuccess)
      return NH_E_CUDA;
    const DTensor *gs = cache.gate_slots(), *us = cache.up_slots(), *ds = cache.down_slots();
    NhGroupedRowDot g;
    std::memset(&g, 0, sizeof(g));
    g.w = gs->data;
    g.w2 = us->data;
    g.mstride = gs->nb[2];
    g.mstride2 = us->nb[2];
    g.type = gs->type;
    g.type2 = us->type;
    g.n = d;
    g.rows = F;
    g.n_groups = slots;
    g.off = off;
    g.cnt = cnt;
    g.act_idx = act_idx;
    g.out_idx = out_idx;
    g.max_tokens = B;
    g.q8 = q8;
    g.out = ff;
    g.out_stride = F;
    g.mode = NH_ROWDOT_SWIGLU;
    NH_B_TRY(nh_batch_rowdot(&g, s));
    NH_B_TRY(nh_batch_prep(ff, F, BK, nullptr, c.rms_eps, 0, F, q8ff, nullptr, s));
    std::memset(&g, 0, sizeof(g));
    g.w = ds->data;
    g.mstride = ds->nb[2];
    g.type = ds->type;
    g.type2 = ds->type;
    g.n = F;
    g.rows = d;
    g.n_groups = slots;
    g.off = off;
    g.cnt = cnt;
    g.act_idx = out_idx;
    g.out_idx = out_idx;
    g.max_tokens = B;
    g.q8 = q8ff;
    g.out = y;
    g.out_stride = d;
    g.mode = NH_ROWDOT_STORE;
    NH_B_TRY(nh_batch_rowdot(&g, s));
    NH_B_TRY(cache.Commit(s));
  }
  se.waves += n_waves;
  se.host_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  return NH_OK;
}

}  // namespace

std::vector<std::vector<int32_t>> GreedyGenerateCachedBatch(const OlmoeModel& model,
                                                            const std::vector<std::vector<int32_t>>& prompts,
                                                            int n_predict, bool norm_topk, BatchOptions* opt) {
  BatchOptions local;
  BatchOptions& o = opt != nullptr ? *opt : local;
  o.status = NH_OK;
  if (prompts.empty() || n_predict <= 0) return {};
  const OlmoeConfig& c = model.config();
  o.status = CheckPrompts(prompts, c);
  if (o.status != NH_OK) return {};
  ModelView m;
  if (!BuildView(model, true, &m)) {
    o.status = NH_E_STATE;
    return {};
  }
  // Expert parallelism: this rank owns experts [shard.first, +count) and the
  // sequences given here; all ranks' tokens meet at every MoE layer.
  const ExpertGroup* ep = o.ep;
  const int W = ep != nullptr ? ep->world() : 1;
  const ExpertShard shard = ep != nullptr ? ExpertShard::Of(c.n_expert, W, ep->rank()) : ExpertShard{0, c.n_expert};
  if (ep != nullptr && (c.n_expert % W != 0 || !Nccl().ok)) {
    o.status = NH_E_ARG;
    return {};
  }
  // The expert weights of the owned shard: the model holds exactly the shard
  // (its tensors start at expert shard.first) or all experts.
  uint64_t e_skip = 0;
  if (model.holds_all_experts()) {
    e_skip = shard.first;
  } else if (model.expert_first() != shard.first || model.expert_count() != shard.count) {
    o.status = NH_E_STATE;
    return {};
  }
  return RunBatch(m, c, prompts, n_predict, norm_topk, o, shard, e_skip, nullptr);
}

std::vector<std::vector<int32_t>> StreamingGenerateBatch(const StreamingModel& model,
                                                         const std::vector<std::vector<int32_t>>& prompts,
                                                         int n_predict, bool norm_topk, int capacity,
                                                         const StreamingOptions& opt, BatchOptions* bopt) {
  BatchOptions local;
  BatchOptions& o = bopt != nullptr ? *bopt : local;
  StreamingStats local_stats;
  StreamingStats& stats = opt.stats != nullptr ? *opt.stats : local_stats;
  o.status = stats.status = NH_OK;
  if (prompts.empty() || n_predict <= 0) return {};
  const OlmoeConfig& c = model.config();
  StreamingModel::Workspace* ws = model.workspace();
  o.status = ws == nullptr || !ws->view_ok ? NH_E_STATE : capacity <= 0 ? NH_E_ARG : CheckPrompts(prompts, c);
  // Expert parallelism: this GPU streams only its shard's experts through its
  // own `capacity` slots per layer and serves every rank's picks of them.
  const ExpertGroup* ep = o.ep;
  const int W = ep != nullptr ? ep->world() : 1;
  const ExpertShard shard = ep != nullptr ? ExpertShard::Of(c.n_expert, W, ep->rank()) : ExpertShard{0, c.n_expert};
  if (ep != nullptr && (c.n_expert % W != 0 || !Nccl().ok)) o.status = NH_E_ARG;
  if (o.status != NH_OK) {
    stats.status = o.status;
    return {};
  }
  const int L = static_cast<int>(c.n_layers);
  std::vector<std::unique_ptr<ExpertSlotCache>> owned;
  StreamedExperts se;
  se.copy_stream = ws->copy_stream;
  se.shard = shard;
  const uint32_t pin_slots =
      opt.pin_slots > 0 ? opt.pin_slots : LearnedPinSlots(static_cast<uint32_t>(capacity));
  // Learned pin chooses among the served experts only.
  UsageHistogram shard_usage;
  const UsageHistogram* usage = opt.usage;
  if (usage != nullptr && W > 1) {
    shard_usage.per_layer.resize(usage->per_layer.size());
    for (size_t l = 0; l < usage->per_layer.size(); ++l)
      for (const auto& kv : usage->per_layer[l])
        if (kv.first >= shard.first && kv.first < shard.first + shard.count) shard_usage.per_layer[l].insert(kv);
    usage = &shard_usage;
  }
  for (int l = 0; l < L; ++l) {
    SlotCacheOptions so;
    so.policy = opt.policy;
    so.usage = usage;
    so.pin_slots = std::min<uint32_t>(pin_slots, static_cast<uint32_t>(capacity));
    so.copy_stream = ws->copy_stream;
    owned.push_back(ExpertSlotCache::Create(c, l, capacity, model.reader(), model.host_store(l), so));
    if (owned.back() == nullptr) {
      o.status = stats.status = NH_E_NOMEM;
      return {};
    }
    se.caches.push_back(owned.back().get());
  }
  auto out = RunBatch(ws->view, c, prompts, n_predict, norm_topk, o, shard, 0, &se);
  cudaStreamSynchronize(ws->copy_stream);
  stats.hits.assign(L, 0);
  stats.misses.assign(L, 0);
  stats.h2d_bytes = 0;
  for (int l = 0; l < L; ++l) {
    stats.hits[l] = owned[l]->hits();
    stats.misses[l] = owned[l]->misses();
    stats.h2d_bytes += owned[l]->h2d_bytes();
  }
  stats.fill_ms = se.host_ms;
  stats.waves = se.waves;
  stats.status = o.status;
  return out;
}

}  // namespace nuthatch

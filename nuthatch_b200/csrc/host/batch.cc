// Batched greedy decode: GreedyGenerateCachedBatch (no reference
// counterpart; the batched form of generate.cc:55-106 that the survey's
// boundary calls for).  B sequences of equal prompt length advance one
// position per step in lockstep; every step is one sequence of kernel
// launches (nh_batch_* in nh_kernels.h), captured once as a CUDA graph and
// replayed.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

#include "engine.h"
#include "nccl_api.h"
#include "nuthatch/expert_parallel.h"
#include "nuthatch/generate.h"
#include "nuthatch/gguf_file.h"

namespace nuthatch {

namespace {

// Device buffers of one batched generation.
class BatchBuffers {
 public:
  ~BatchBuffers() {
    for (void* p : owned_) cudaFree(p);
    if (graph_ != nullptr) cudaGraphExecDestroy(graph_);
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
  bool ok_ = true;
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_ = nullptr;

 private:
  std::vector<void*> owned_;
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

}  // namespace

std::vector<std::vector<int32_t>> GreedyGenerateCachedBatch(const OlmoeModel& model,
                                                            const std::vector<std::vector<int32_t>>& prompts,
                                                            int n_predict, bool norm_topk, BatchOptions* opt) {
  BatchOptions local;
  BatchOptions& o = opt != nullptr ? *opt : local;
  o.status = NH_OK;
  std::vector<std::vector<int32_t>> out;
  const int B = static_cast<int>(prompts.size());
  if (B == 0 || n_predict <= 0) return out;
  const int P = static_cast<int>(prompts[0].size());
  const OlmoeConfig& c = model.config();
  for (const auto& p : prompts) {
    if (static_cast<int>(p.size()) != P || P == 0) {
      o.status = NH_E_ARG;
      return out;
    }
    for (int32_t t : p)
      if (t < 0 || static_cast<uint32_t>(t) >= c.n_vocab) {
        o.status = NH_E_ARG;
        return out;
      }
  }
  ModelView m;
  if (!BuildView(model, true, &m)) {
    o.status = NH_E_STATE;
    return out;
  }
  const int64_t d = c.n_embd, hd = c.head_dim(), dkv = static_cast<int64_t>(c.n_head_kv) * hd, F = c.n_ff,
                E = c.n_expert, K = c.n_expert_used, V = c.n_vocab, L = c.n_layers;
  // Expert parallelism: this rank owns experts [shard.first, +count) and the
  // B sequences given here; all W ranks' tokens meet at every MoE layer.
  const ExpertGroup* ep = o.ep;
  const int W = ep != nullptr ? ep->world() : 1;
  const ExpertShard shard = ep != nullptr ? ExpertShard::Of(c.n_expert, W, ep->rank()) : ExpertShard{0, c.n_expert};
  if (ep != nullptr && (c.n_expert % W != 0 || !Nccl().ok)) {
    o.status = NH_E_ARG;
    return out;
  }
  // The expert weights of the owned shard: the model holds exactly the shard
  // (its tensors start at expert shard.first) or all experts.
  uint64_t e_skip = 0;
  if (model.holds_all_experts()) {
    e_skip = shard.first;
  } else if (model.expert_first() != shard.first || model.expert_count() != shard.count) {
    o.status = NH_E_STATE;
    return out;
  }
  const int max_seq = P + n_predict;
  const int BK = B * static_cast<int>(K);
  const int BW = B * W, BKW = BK * W;  // rows of every rank's tokens / picks
  BatchBuffers bb;
  NhDecodeState* state = bb.Alloc<NhDecodeState>(1);
  int32_t* prm = bb.Alloc<int32_t>(static_cast<size_t>(B) * P);
  int32_t* fed = bb.Alloc<int32_t>(B);
  int32_t* outs = bb.Alloc<int32_t>(static_cast<size_t>(B) * n_predict);
  float* h = bb.Alloc<float>(B * d);
  float* q = bb.Alloc<float>(B * d);
  float* kk = bb.Alloc<float>(B * dkv);
  float* v = bb.Alloc<float>(B * dkv);
  float* qr = bb.Alloc<float>(B * d);
  float* att = bb.Alloc<float>(B * d);
  float* xn = bb.Alloc<float>(B * d);
  const int64_t q8_row = nh_batch_q8_bytes(1, d);
  uint8_t* q8 = bb.Alloc<uint8_t>(q8_row * B);
  int32_t* sel = bb.Alloc<int32_t>(BK);
  float* wts = bb.Alloc<float>(BK);
  int32_t* off = bb.Alloc<int32_t>(E);
  int32_t* cnt = bb.Alloc<int32_t>(E);
  int32_t* act_idx = bb.Alloc<int32_t>(BKW);
  int32_t* out_idx = bb.Alloc<int32_t>(BKW);
  float* ff = bb.Alloc<float>(static_cast<size_t>(BKW) * F);
  uint8_t* q8ff = bb.Alloc<uint8_t>(nh_batch_q8_bytes(BKW, F));
  float* y = bb.Alloc<float>(static_cast<size_t>(BKW) * d);
  // Expert-parallel exchange buffers: every rank's activation rows and
  // selections (all-gathered), and the pick rows returned by each rank.
  uint8_t* q8_all = W > 1 ? bb.Alloc<uint8_t>(q8_row * BW) : q8;
  int32_t* sel_all = W > 1 ? bb.Alloc<int32_t>(BKW) : sel;
  float* y_recv = W > 1 ? bb.Alloc<float>(static_cast<size_t>(BKW) * d) : y;
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
  bool setup = cudaMemcpy(prm, flat.data(), flat.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemcpy(rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemcpy(state, &st0, sizeof(st0), cudaMemcpyHostToDevice) == cudaSuccess &&
               cudaMemset(attn_scratch, 0, attn_bytes) == cudaSuccess && cudaMemset(ticket, 0, 64) == cudaSuccess &&
               cudaMemset(fed, 0, B * 4) == cudaSuccess &&
               cudaMemset(ff, 0, static_cast<size_t>(BKW) * F * 4) == cudaSuccess &&
               cudaMemset(y, 0, static_cast<size_t>(BKW) * d * 4) == cudaSuccess &&
               cudaMemset(y_recv, 0, static_cast<size_t>(BKW) * d * 4) == cudaSuccess &&
               cudaDeviceSynchronize() == cudaSuccess &&
               cudaStreamCreateWithFlags(&bb.stream_, cudaStreamNonBlocking) == cudaSuccess;
  if (!setup) {
    o.status = NH_E_CUDA;
    return out;
  }
  cudaStream_t s = bb.stream_;
  const float eps = c.rms_eps;
  const float kq_scale = 1.0f / std::sqrt(static_cast<float>(hd));

  auto dense = [&](const void* w, int32_t type, int64_t rows, int64_t n, const void* act, float* o_, int64_t stride,
                   int mode) {
    NhGroupedRowDot g;
    std::memset(&g, 0, sizeof(g));
    g.w = w;
    g.type = type;
    g.type2 = type;
    g.n = n;
    g.rows = rows;
    g.n_groups = 1;
    g.n_tok = B;
    g.max_tokens = B;
    g.q8 = act;
    g.out = o_;
    g.out_stride = stride;
    g.mode = mode;
    return nh_batch_rowdot(&g, s);
  };
  auto step = [&]() -> int {
    NH_B_TRY(nh_batch_embed(state, prm, P, fed, B, m.embd, m.te, d, V, h, s));
    for (int l = 0; l < static_cast<int>(L); ++l) {
      const LayerView& Lv = m.layers[l];
      float* kc = kv + static_cast<size_t>(2 * l) * B * max_seq * dkv;
      float* vc = kv + static_cast<size_t>(2 * l + 1) * B * max_seq * dkv;
      NH_B_TRY(nh_batch_prep(h, d, B, Lv.attn_norm, eps, 1, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wq, Lv.tq, d, d, q8, q, d, NH_ROWDOT_STORE));
      NH_B_TRY(dense(Lv.wk, Lv.tk, dkv, d, q8, kk, dkv, NH_ROWDOT_STORE));
      NH_B_TRY(dense(Lv.wv, Lv.tv, dkv, d, q8, v, dkv, NH_ROWDOT_STORE));
      NH_B_TRY(nh_batch_qk(state, q, kk, v, Lv.q_norm, Lv.k_norm, eps, B, c.n_head, c.n_head_kv,
                           static_cast<int>(hd), rope, kc, vc, max_seq, qr, s));
      NH_B_TRY(nh_batch_attention(state, qr, B, c.n_head, c.n_head_kv, static_cast<int>(hd), kq_scale, kc, vc,
                                  max_seq, attn_scratch, att, s));
      NH_B_TRY(nh_batch_prep(att, d, B, nullptr, eps, 0, d, q8, nullptr, s));
      NH_B_TRY(dense(Lv.wo, Lv.to, d, d, q8, h, d, NH_ROWDOT_RESIDUAL));
      NH_B_TRY(nh_batch_prep(h, d, B, Lv.ffn_norm, eps, 1, d, q8, xn, s));
      NH_B_TRY(nh_batch_router(xn, Lv.router, B, d, static_cast<int>(E), static_cast<int>(K), norm_topk ? 1 : 0,
                               sel, wts, s));
      if (W > 1) NH_B_TRY(ExchangeTokens(*ep, q8, q8_row * B, q8_all, sel, BK, sel_all, s));
      // The owned experts over every rank's tokens: token j of the
      // gathered rows is rank j / B's sequence j % B.
      NH_B_TRY(nh_batch_moe_plan_range(sel_all, BW, static_cast<int>(K), static_cast<int>(shard.first),
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
      g.max_tokens = BW;
      g.q8 = q8_all;
      g.out = ff;
      g.out_stride = F;
      g.mode = NH_ROWDOT_SWIGLU;
      NH_B_TRY(nh_batch_rowdot(&g, s));
      NH_B_TRY(nh_batch_prep(ff, F, BKW, nullptr, eps, 0, F, q8ff, nullptr, s));
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
      g.act_idx = out_idx;  // the ff row of pair j is its (token, slot) index
      g.out_idx = out_idx;
      g.max_tokens = BW;
      g.q8 = q8ff;
      g.out = y;
      g.out_stride = d;
      g.mode = NH_ROWDOT_STORE;
      NH_B_TRY(nh_batch_rowdot(&g, s));
      if (W > 1) {
        // Rows of rank r's picks go back to rank r; the combine takes each
        // pick's row from the block of the rank that owns its expert.
        NH_B_TRY(ReturnPicks(*ep, y, static_cast<size_t>(BK) * d, y_recv, s));
        NH_B_TRY(nh_ep_combine(y_recv, static_cast<int64_t>(BK) * d, W, sel, wts, B, static_cast<int>(K), d,
                               static_cast<int>(shard.count), h, s));
      } else {
        NH_B_TRY(nh_batch_combine(y, wts, B, static_cast<int>(K), d, h, s));
      }
    }
    NH_B_TRY(nh_batch_prep(h, d, B, m.out_norm, eps, 1, d, q8, nullptr, s));
    NH_B_TRY(dense(m.out, m.tout, V, d, q8, logits, V, NH_ROWDOT_STORE));
    return nh_batch_argmax(state, logits, B, V, fed, outs, n_predict, ticket, s);
  };

  const int steps = P + n_predict - 1;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEventCreate(&ev0);
  cudaEventCreate(&ev1);
  int rc = NH_OK;
  for (int t = 0; t < steps && rc == NH_OK; ++t) {
    if (t == P - 1) cudaEventRecord(ev0, s);  // decode: from the last prompt position on
    if (t == 0 || !o.use_graph) {
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

}  // namespace nuthatch

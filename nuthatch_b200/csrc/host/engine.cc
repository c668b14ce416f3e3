// Device workspace and per-token kernel sequence.
#include "engine.h"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>

#include "nuthatch/gguf_file.h"
#include "nuthatch/streaming_model.h"

namespace nuthatch {

namespace {

template <typename T>
int DevAlloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  return cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)) == cudaSuccess ? NH_OK : NH_E_NOMEM;
}
template <typename T>
int HostAlloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  return cudaHostAlloc(reinterpret_cast<void**>(p), count * sizeof(T), cudaHostAllocDefault) == cudaSuccess
             ? NH_OK
             : NH_E_NOMEM;
}
// Resident steps run each layer's MoE block as one cooperative kernel unless
// NH_FUSED_MOE=0 (read once; both forms give identical results).
bool FusedMoeEnabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("NH_FUSED_MOE");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v != 0;
}

template <typename T>
void DevFree(T*& p) {
  if (p != nullptr) cudaFree(p);
  p = nullptr;
}
// Pinned host memory the device can address (for flags and small hand-overs).
template <typename T>
int MappedAlloc(T** host, T** dev, size_t count) {
  *host = nullptr;
  *dev = nullptr;
  if (cudaHostAlloc(reinterpret_cast<void**>(host), std::max<size_t>(count, 1) * sizeof(T), cudaHostAllocMapped) !=
      cudaSuccess)
    return NH_E_NOMEM;
  std::memset(*host, 0, std::max<size_t>(count, 1) * sizeof(T));
  return cudaHostGetDevicePointer(reinterpret_cast<void**>(dev), *host, 0) == cudaSuccess ? NH_OK : NH_E_CUDA;
}

template <typename T>
void HostFree(T*& p) {
  if (p != nullptr) cudaFreeHost(p);
  p = nullptr;
}

#define NH_TRY(expr)              \
  do {                            \
    const int rc__ = (expr);      \
    if (rc__ != NH_OK) return rc__; \
  } while (0)

}  // namespace

uint32_t HeldExperts(const OlmoeModel& m) { return m.expert_count(); }
uint32_t HeldExperts(const StreamingModel& m) { return m.config().n_expert; }

template <typename M>
bool BuildView(const M& m, bool experts, ModelView* v) {
  const OlmoeConfig& c = m.config();
  v->cfg = c;
  const int64_t d = c.n_embd, dkv = static_cast<int64_t>(c.n_head_kv) * c.head_dim();
  if (c.n_layers == 0 || d == 0 || c.n_head == 0 || c.n_head_kv == 0 || c.n_ff == 0 || c.n_expert == 0 ||
      c.n_expert_used == 0 || c.n_expert_used > c.n_expert || c.n_vocab == 0 || d % c.n_head != 0 ||
      c.n_head % c.n_head_kv != 0)
    return false;
  auto need = [&](const DTensor* t, int64_t ne0, int64_t ne1, int64_t ne2) {
    return t != nullptr && t->ne[0] == ne0 && t->ne[1] == ne1 && t->ne[2] == ne2;
  };
  const DTensor* emb = m.tensor("token_embd.weight");
  const DTensor* on = m.tensor("output_norm.weight");
  const DTensor* out = m.tensor("output.weight");
  if (!need(emb, d, c.n_vocab, 1) || !need(on, d, 1, 1) || !need(out, d, c.n_vocab, 1)) return false;
  if (on->type != kTypeF32) return false;
  v->embd = emb->data;
  v->te = emb->type;
  v->out_norm = static_cast<const float*>(on->data);
  v->out = out->data;
  v->tout = out->type;
  v->layers.assign(c.n_layers, LayerView());
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    LayerView& L = v->layers[l];
    auto T = [&](const char* s) { return m.layer_tensor(static_cast<int>(l), s); };
    const DTensor *an = T("attn_norm.weight"), *wq = T("attn_q.weight"), *wk = T("attn_k.weight"),
                  *wv = T("attn_v.weight"), *wo = T("attn_output.weight"), *qn = T("attn_q_norm.weight"),
                  *kn = T("attn_k_norm.weight"), *fn = T("ffn_norm.weight"), *r = T("ffn_gate_inp.weight");
    if (!need(an, d, 1, 1) || !need(wq, d, d, 1) || !need(wk, d, dkv, 1) || !need(wv, d, dkv, 1) ||
        !need(wo, d, d, 1) || !need(qn, d, 1, 1) || !need(kn, dkv, 1, 1) || !need(fn, d, 1, 1) ||
        !need(r, d, c.n_expert, 1))
      return false;
    if (an->type != kTypeF32 || qn->type != kTypeF32 || kn->type != kTypeF32 || fn->type != kTypeF32 ||
        r->type != kTypeF32)
      return false;
    L.attn_norm = static_cast<const float*>(an->data);
    L.wq = wq->data;
    L.tq = wq->type;
    L.wk = wk->data;
    L.tk = wk->type;
    L.wv = wv->data;
    L.tv = wv->type;
    L.wo = wo->data;
    L.to = wo->type;
    L.q_norm = static_cast<const float*>(qn->data);
    L.k_norm = static_cast<const float*>(kn->data);
    L.ffn_norm = static_cast<const float*>(fn->data);
    L.router = static_cast<const float*>(r->data);
    if (experts) {
      const DTensor *g = T("ffn_gate_exps.weight"), *u = T("ffn_up_exps.weight"), *dn = T("ffn_down_exps.weight");
      const int64_t ne = HeldExperts(m);
      if (!need(g, d, c.n_ff, ne) || !need(u, d, c.n_ff, ne) || !need(dn, c.n_ff, d, ne)) return false;
      L.gate = g->data;
      L.tg = g->type;
      L.gate_nb2 = g->nb[2];
      L.up = u->data;
      L.tu = u->type;
      L.up_nb2 = u->nb[2];
      L.down = dn->data;
      L.td = dn->type;
      L.down_nb2 = dn->nb[2];
    }
  }
  return true;
}

template bool BuildView<OlmoeModel>(const OlmoeModel&, bool, ModelView*);
template bool BuildView<StreamingModel>(const StreamingModel&, bool, ModelView*);

Engine::Engine(const OlmoeConfig& cfg) : cfg_(cfg) {
  cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
}

Engine::~Engine() {
  FreeAll();
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

void Engine::FreeAll() {
  if (graph_ != nullptr) cudaGraphExecDestroy(graph_);
  graph_ = nullptr;
  graph_key_ = ~0ull;
  kv_.reset();
  DevFree(state_);
  HostFree(state_host_);
  HostFree(state_saved_);
  DevFree(prompt_);
  HostFree(prompt_host_);
  DevFree(out_);
  HostFree(out_host_);
  DevFree(h_);
  DevFree(q_);
  DevFree(k_);
  DevFree(v_);
  DevFree(attn_);
  DevFree(sel_);
  DevFree(wsel_);
  HostFree(sel_host_);
  HostFree(wsel_host_);
  HostFree(pub_sel_);
  HostFree(pub_seq_);
  pub_sel_dev_ = nullptr;
  pub_seq_dev_ = nullptr;
  DevFree(wts_);
  DevFree(ff_);
  DevFree(rope_cs_);
  if (attn_scratch_) cudaFree(attn_scratch_);
  if (router_scratch_) cudaFree(router_scratch_);
  if (moe_scratch_) cudaFree(moe_scratch_);
  if (argmax_scratch_) cudaFree(argmax_scratch_);
  attn_scratch_ = router_scratch_ = moe_scratch_ = argmax_scratch_ = nullptr;
  DevFree(trace_sel_);
  DevFree(trace_gap_);
  DevFree(dump_hidden_);
  DevFree(dump_logits_);
  max_seq_ = max_prompt_ = max_predict_ = 0;
}

int Engine::Reserve(int max_seq, int max_prompt, int max_predict, bool dumps) {
  if (max_seq <= 0 || max_prompt <= 0 || max_predict <= 0) return NH_E_ARG;
  if (max_seq <= max_seq_ && max_prompt <= max_prompt_ && max_predict <= max_predict_ && (!dumps || dumps_))
    return NH_OK;
  // Grow geometrically so a sequence of slightly longer requests does not
  // reallocate (and re-capture) every time.
  max_seq = std::max(max_seq, max_seq_ + max_seq_ / 2);
  max_prompt = std::max(max_prompt, max_prompt_);
  max_predict = std::max(max_predict, max_predict_);
  dumps = dumps || dumps_;
  cudaStreamSynchronize(stream_);
  FreeAll();
  const OlmoeConfig& c = cfg_;
  const int64_t d = c.n_embd, dkv = static_cast<int64_t>(c.n_head_kv) * c.head_dim();
  const int64_t L = c.n_layers, K = c.n_expert_used, hd = c.head_dim();
  kv_.reset(new KvCache(c, max_seq));
  if (!kv_->ok()) return NH_E_NOMEM;
  NH_TRY(DevAlloc(&state_, 1));
  NH_TRY(HostAlloc(&state_host_, 1));
  NH_TRY(HostAlloc(&state_saved_, 1));
  NH_TRY(DevAlloc(&prompt_, max_prompt));
  NH_TRY(HostAlloc(&prompt_host_, max_prompt));
  NH_TRY(DevAlloc(&out_, max_predict));
  NH_TRY(HostAlloc(&out_host_, max_predict));
  NH_TRY(DevAlloc(&h_, d));
  NH_TRY(DevAlloc(&q_, d));
  NH_TRY(DevAlloc(&k_, dkv));
  NH_TRY(DevAlloc(&v_, dkv));
  NH_TRY(DevAlloc(&attn_, d));
  NH_TRY(DevAlloc(&sel_, K));
  NH_TRY(DevAlloc(&wsel_, K));
  NH_TRY(HostAlloc(&sel_host_, K));
  NH_TRY(HostAlloc(&wsel_host_, K));
  NH_TRY(MappedAlloc(&pub_sel_, &pub_sel_dev_, K));
  NH_TRY(MappedAlloc(&pub_seq_, &pub_seq_dev_, 1));
  *pub_seq_ = pub_count_;
  NH_TRY(DevAlloc(&wts_, K));
  NH_TRY(DevAlloc(&ff_, K * c.n_ff));
  std::vector<float> cs(static_cast<size_t>(max_seq) * hd);
  nh_rope_table(c.rope_freq_base, static_cast<int>(hd), max_seq, cs.data());
  NH_TRY(DevAlloc(&rope_cs_, cs.size()));
  if (cudaMemcpy(rope_cs_, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return NH_E_CUDA;
  const int64_t ab = nh_attention_scratch_bytes(c.n_head, static_cast<int>(hd), max_seq);
  const int64_t rb = nh_router_scratch_bytes(c.n_expert);
  const int64_t mb = nh_argmax_scratch_bytes(c.n_vocab);
  const int64_t fb = nh_moe_layer_scratch_bytes(c.n_expert);
  if (cudaMalloc(&attn_scratch_, ab) != cudaSuccess || cudaMalloc(&router_scratch_, rb) != cudaSuccess ||
      cudaMalloc(&moe_scratch_, fb) != cudaSuccess || cudaMalloc(&argmax_scratch_, mb) != cudaSuccess)
    return NH_E_NOMEM;
  cudaMemset(attn_scratch_, 0, ab);
  cudaMemset(router_scratch_, 0, rb);
  cudaMemset(moe_scratch_, 0, fb);
  cudaMemset(argmax_scratch_, 0, mb);
  NH_TRY(DevAlloc(&trace_sel_, static_cast<size_t>(max_seq) * L * K));
  NH_TRY(DevAlloc(&trace_gap_, static_cast<size_t>(max_seq) * L));
  if (dumps) {
    NH_TRY(DevAlloc(&dump_hidden_, static_cast<size_t>(max_predict) * L * d));
    NH_TRY(DevAlloc(&dump_logits_, static_cast<size_t>(max_predict) * c.n_vocab));
  }
  max_seq_ = max_seq;
  max_prompt_ = max_prompt;
  max_predict_ = max_predict;
  dumps_ = dumps;
  ++alloc_gen_;
  return cudaDeviceSynchronize() == cudaSuccess ? NH_OK : NH_E_CUDA;
}

int Engine::Begin(const int32_t* prompt, int n_prompt, int n_predict, int start_pos) {
  if (n_prompt <= 0 || n_prompt > max_prompt_ || n_predict <= 0 || n_predict > max_predict_ ||
      n_prompt + n_predict > max_seq_)
    return NH_E_CAPACITY;
  if (start_pos < 0 || start_pos >= n_prompt) return NH_E_ARG;
  std::memcpy(prompt_host_, prompt, static_cast<size_t>(n_prompt) * 4);
  *state_host_ = NhDecodeState{start_pos, n_prompt, n_predict, 0, 0, 0, 0, 0};
  if (cudaMemcpyAsync(prompt_, prompt_host_, static_cast<size_t>(n_prompt) * 4, cudaMemcpyHostToDevice,
                      stream_) != cudaSuccess ||
      cudaMemcpyAsync(state_, state_host_, sizeof(NhDecodeState), cudaMemcpyHostToDevice, stream_) != cudaSuccess)
    return NH_E_CUDA;
  return NH_OK;
}

int Engine::EnqueueEmbed(const ModelView& m) {
  return nh_embed_step(state_, prompt_, m.embd, m.te, cfg_.n_embd, cfg_.n_vocab, h_, stream_);
}

int Engine::EnqueueAttention(const ModelView& m, int l) {
  const OlmoeConfig& c = cfg_;
  const LayerView& L = m.layers[l];
  const int64_t dkv = static_cast<int64_t>(c.n_head_kv) * c.head_dim();
  const int hd = static_cast<int>(c.head_dim());
  const float kq_scale = 1.0f / std::sqrt(static_cast<float>(hd));
  NH_TRY(nh_qkv_proj(state_, h_, L.attn_norm, c.rms_eps, L.wq, L.tq, L.wk, L.tk, L.wv, L.tv, c.n_embd, dkv, q_, k_,
                     v_, stream_));
  NH_TRY(nh_attention_step(state_, q_, k_, v_, L.q_norm, L.k_norm, c.rms_eps, c.n_head, c.n_head_kv, hd, rope_cs_,
                           kq_scale, kv_->k(l), kv_->v(l), max_seq_, attn_scratch_, attn_, stream_));
  return nh_out_proj_residual(state_, attn_, L.wo, L.to, c.n_embd, h_, stream_);
}

void Engine::FillMoeLayer(const ModelView& m, int l, bool norm_topk, bool trace, bool dumps, NhMoeLayer* out) {
  const OlmoeConfig& c = cfg_;
  const LayerView& L = m.layers[l];
  NhMoeLayer& a = *out;
  a = NhMoeLayer{};
  a.state = state_;
  a.h = h_;
  a.ffn_norm = L.ffn_norm;
  a.eps = c.rms_eps;
  a.router = L.router;
  a.n_embd = c.n_embd;
  a.n_ff = c.n_ff;
  a.n_expert = static_cast<int>(c.n_expert);
  a.k = static_cast<int>(c.n_expert_used);
  a.norm_topk = norm_topk ? 1 : 0;
  a.layer = l;
  a.n_layers = static_cast<int>(c.n_layers);
  a.gate = L.gate;
  a.tg = L.tg;
  a.gate_nb2 = L.gate_nb2;
  a.up = L.up;
  a.tu = L.tu;
  a.up_nb2 = L.up_nb2;
  a.down = L.down;
  a.td = L.td;
  a.down_nb2 = L.down_nb2;
  a.sel = sel_;
  a.wts = wts_;
  a.trace_sel = trace ? trace_sel_ : nullptr;
  a.trace_gap = trace ? trace_gap_ : nullptr;
  a.ff = ff_;
  a.dump = dumps ? dump_hidden_ : nullptr;
  a.dump_step_stride = static_cast<int64_t>(c.n_layers) * c.n_embd;
  a.dump_offset = l * c.n_embd;
  a.scratch = moe_scratch_;
}

int Engine::EnqueueFusedMoe(const ModelView& m, int l, bool norm_topk, bool trace, bool dumps) {
  NhMoeLayer a;
  FillMoeLayer(m, l, norm_topk, trace, dumps, &a);
  return nh_moe_layer(&a, stream_);
}

int Engine::EnqueueAttnPhase(const ModelView& m, int l, bool norm_topk, bool trace) {
  const OlmoeConfig& c = cfg_;
  const LayerView& L = m.layers[l];
  NH_TRY(EnqueueAttention(m, l));
  return nh_router_topk(state_, h_, L.ffn_norm, c.rms_eps, L.router, c.n_embd, c.n_expert, c.n_expert_used,
                        norm_topk ? 1 : 0, sel_, wts_, trace ? trace_sel_ : nullptr, trace ? trace_gap_ : nullptr, l,
                        c.n_layers, router_scratch_, stream_);
}

int Engine::AwaitSelection(double timeout_s) {
  const int K = static_cast<int>(cfg_.n_expert_used);
  const uint32_t seq = ++pub_count_;
  NH_TRY(nh_publish_selection(sel_, K, pub_sel_dev_, pub_seq_dev_, seq, stream_));
  const volatile uint32_t* flag = pub_seq_;
  const auto t0 = std::chrono::steady_clock::now();
  for (uint64_t spins = 0; *flag != seq; ++spins) {
    if ((spins & 4095) == 4095 &&
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
      // A failed launch never publishes: report the stream's error if any.
      return cudaStreamSynchronize(stream_) != cudaSuccess ? NH_E_CUDA : NH_E_TIMEOUT;
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  const volatile int32_t* ids = pub_sel_;
  for (int i = 0; i < K; ++i) sel_host_[i] = ids[i];
  return NH_OK;
}

int Engine::EnqueueMoePhase(const ModelView& m, int l, const void* gate, int32_t tg, uint64_t gnb2, const void* up,
                            int32_t tu, uint64_t unb2, const void* down, int32_t td, uint64_t dnb2,
                            const int32_t* wsel, bool dumps, const int32_t* slots_host) {
  const OlmoeConfig& c = cfg_;
  const LayerView& L = m.layers[l];
  const int64_t d = c.n_embd;
  float* dump = dumps ? dump_hidden_ : nullptr;
  const int64_t dstride = static_cast<int64_t>(c.n_layers) * d;
  // gate/up also starts this layer's selected down slices towards L2.
  if (slots_host != nullptr) {
    NH_TRY(nh_moe_gate_up_slots(state_, h_, L.ffn_norm, c.rms_eps, slots_host, c.n_expert_used, gate, tg, gnb2, up,
                                tu, unb2, c.n_embd, c.n_ff, ff_, down, dnb2, stream_));
    return nh_moe_down_combine_slots(state_, ff_, slots_host, wts_, c.n_expert_used, down, td, dnb2, c.n_ff, d, h_,
                                     dump, dstride, l * d, stream_);
  }
  NH_TRY(nh_moe_gate_up_prefetch(state_, h_, L.ffn_norm, c.rms_eps, wsel, c.n_expert_used, gate, tg, gnb2, up, tu,
                                 unb2, c.n_embd, c.n_ff, ff_, down, dnb2, stream_));
  return nh_moe_down_combine(state_, ff_, wsel, wts_, c.n_expert_used, down, td, dnb2, c.n_ff, d, h_, dump, dstride,
                             l * d, stream_);
}

int Engine::EnqueueFinal(const ModelView& m, bool dumps) {
  return nh_lm_head_argmax(state_, h_, m.out_norm, cfg_.rms_eps, m.out, m.tout, cfg_.n_embd, cfg_.n_vocab, out_,
                           dumps ? dump_logits_ : nullptr, argmax_scratch_, stream_);
}

int Engine::EnqueueStep(const ModelView& m, bool norm_topk, bool trace, bool dumps) {
  NH_TRY(EnqueueEmbed(m));
  int launches = 2;  // embed, lm_head
  for (int l = 0; l < static_cast<int>(cfg_.n_layers); ++l) {
    const LayerView& L = m.layers[l];
    launches += 6;
    if (FusedMoeEnabled()) {
      NH_TRY(EnqueueAttention(m, l));
      const int rc = EnqueueFusedMoe(m, l, norm_topk, trace, dumps);
      if (rc == NH_OK) {
        launches -= 2;
        continue;
      }
      if (rc != NH_E_ARG && rc != NH_E_TYPE) return rc;
      // Shapes outside the fused kernel: router, gate/up and down separately.
      const OlmoeConfig& c = cfg_;
      NH_TRY(nh_router_topk(state_, h_, L.ffn_norm, c.rms_eps, L.router, c.n_embd, c.n_expert, c.n_expert_used,
                            norm_topk ? 1 : 0, sel_, wts_, trace ? trace_sel_ : nullptr,
                            trace ? trace_gap_ : nullptr, l, c.n_layers, router_scratch_, stream_));
    } else {
      NH_TRY(EnqueueAttnPhase(m, l, norm_topk, trace));
    }
    NH_TRY(EnqueueMoePhase(m, l, L.gate, L.tg, L.gate_nb2, L.up, L.tu, L.up_nb2, L.down, L.td, L.down_nb2, sel_,
                           dumps));
  }
  NH_TRY(EnqueueFinal(m, dumps));
  step_launches_ = launches;
  return NH_OK;
}

int Engine::RunSteps(const ModelView& m, int steps, bool norm_topk, bool trace, bool dumps, bool use_graph) {
  if (steps <= 0) return NH_OK;
  if (!use_graph) {
    for (int s = 0; s < steps; ++s) NH_TRY(EnqueueStep(m, norm_topk, trace, dumps));
    return NH_OK;
  }
  const uint64_t key = (alloc_gen_ << 3) | (norm_topk ? 1u : 0u) | (trace ? 2u : 0u) | (dumps ? 4u : 0u);
  int done = 0;
  if (graph_ == nullptr || graph_key_ != key) {
    // One eager step first: it configures the kernels' shared-memory limits
    // outside of stream capture.
    NH_TRY(EnqueueStep(m, norm_topk, trace, dumps));
    done = 1;
    if (graph_ != nullptr) cudaGraphExecDestroy(graph_);
    graph_ = nullptr;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return NH_E_CUDA;
    const int rc = EnqueueStep(m, norm_topk, trace, dumps);
    const cudaError_t ec = cudaStreamEndCapture(stream_, &g);
    if (rc != NH_OK || ec != cudaSuccess) {
      if (g != nullptr) cudaGraphDestroy(g);
      return rc != NH_OK ? rc : NH_E_CUDA;
    }
    const cudaError_t ei = cudaGraphInstantiate(&graph_, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
      graph_ = nullptr;
      return NH_E_CUDA;
    }
    graph_key_ = key;
  }
  for (int s = done; s < steps; ++s) {
    if (cudaGraphLaunch(graph_, stream_) != cudaSuccess) return NH_E_CUDA;
  }
  return NH_OK;
}

int Engine::SaveState() {
  if (state_ == nullptr) return NH_E_STATE;
  if (cudaMemcpyAsync(state_saved_, state_, sizeof(NhDecodeState), cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
      cudaStreamSynchronize(stream_) != cudaSuccess)
    return NH_E_CUDA;
  return NH_OK;
}

int Engine::RestoreState() {
  if (state_ == nullptr) return NH_E_STATE;
  return cudaMemcpyAsync(state_, state_saved_, sizeof(NhDecodeState), cudaMemcpyHostToDevice, stream_) ==
                 cudaSuccess
             ? NH_OK
             : NH_E_CUDA;
}

int Engine::KernelLoop(const ModelView& m, int which, int reps) {
  const OlmoeConfig& c = cfg_;
  int launches = 0;
  for (int r = 0; r < reps; ++r) {
    for (int l = 0; l < static_cast<int>(c.n_layers); ++l) {
      const LayerView& L = m.layers[l];
      int rc;
      if (which == 0) {
        rc = nh_moe_gate_up(state_, h_,L.ffn_norm, c.rms_eps, sel_, c.n_expert_used, L.gate, L.tg, L.gate_nb2, L.up, L.tu,
                            L.up_nb2, c.n_embd, c.n_ff, ff_, stream_);
      } else if (which == 3) {
        rc = EnqueueFusedMoe(m, l, false, false, false);
      } else if (which == 1) {
        rc = nh_moe_down_combine(state_, ff_, sel_, wts_, c.n_expert_used, L.down, L.td, L.down_nb2, c.n_ff,
                                 c.n_embd, h_, nullptr, 0, 0, stream_);
      } else {
        const int64_t dkv = static_cast<int64_t>(c.n_head_kv) * c.head_dim();
        rc = nh_qkv_proj(state_, h_,L.attn_norm, c.rms_eps, L.wq, L.tq, L.wk, L.tk, L.wv, L.tv, c.n_embd, dkv, q_, k_, v_,
                         stream_);
      }
      if (rc != NH_OK) return rc;
      ++launches;
    }
  }
  return launches;
}

int Engine::Finish(int n_predict, std::vector<int32_t>* out) {
  if (cudaMemcpyAsync(out_host_, out_, static_cast<size_t>(n_predict) * 4, cudaMemcpyDeviceToHost, stream_) !=
          cudaSuccess ||
      cudaMemcpyAsync(state_host_, state_, sizeof(NhDecodeState), cudaMemcpyDeviceToHost, stream_) != cudaSuccess)
    return NH_E_CUDA;
  if (cudaStreamSynchronize(stream_) != cudaSuccess) return NH_E_CUDA;
  if (state_host_->error != 0) return state_host_->error;
  out->assign(out_host_, out_host_ + n_predict);
  return NH_OK;
}

}  // namespace nuthatch

// One-shot prompt prefill for resident generation (reference:
// generate.cc:63-91 forwards the whole prompt as one graph, forward.cc:45-79).
// The prompt positions before the last are processed as a batch of rows of
// one sequence: per layer, RMSNorm + Q8_K activations for all rows, grouped
// row dots for Q/K/V, QK-norm + RoPE + K/V append at each row's position,
// causal prefill attention, the output projection, the router, the per-expert
// token lists and the grouped gate/up and down products, and the top-k-order
// combine.  The last prompt position then runs as the first batch-1 step,
// which forms its logits and the first generated id.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "engine.h"

namespace nuthatch {

namespace {

#define NH_PF_TRY(x)              \
  do {                            \
    const int rc_ = (x);          \
    if (rc_ != NH_OK) return rc_; \
  } while (0)

template <typename T>
int DevAllocN(T** p, size_t count) {
  *p = nullptr;
  return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(T)) == cudaSuccess
             ? NH_OK
             : NH_E_NOMEM;
}

template <typename T>
void DevRelease(T*& p) {
  if (p != nullptr) cudaFree(p);
  p = nullptr;
}

bool QuantType(int32_t t) { return t == NH_TYPE_Q4_K || t == NH_TYPE_Q6_K; }

// Row lengths the grouped row-dot kernels take: 256 x {1, 2, 4, 8}.
bool RowLenOk(int64_t n) {
  if (n < 256 || n % 256 != 0) return false;
  const int64_t g = n / 256;
  return g <= 8 && (g & (g - 1)) == 0;
}

}  // namespace

void PrefillBuffers::Release() {
  DevRelease(h);
  DevRelease(q);
  DevRelease(k);
  DevRelease(v);
  DevRelease(qr);
  DevRelease(att);
  DevRelease(xn);
  DevRelease(wts);
  DevRelease(ff);
  DevRelease(y);
  DevRelease(q8);
  DevRelease(q8ff);
  DevRelease(sel);
  DevRelease(off);
  DevRelease(cnt);
  DevRelease(act_idx);
  DevRelease(out_idx);
  rows = 0;
}

PrefillBuffers::~PrefillBuffers() { Release(); }

int PrefillBuffers::Reserve(const OlmoeConfig& c, int n) {
  if (n <= rows) return NH_OK;
  Release();
  const size_t d = c.n_embd, dkv = static_cast<size_t>(c.n_head_kv) * c.head_dim(), F = c.n_ff, K = c.n_expert_used;
  const size_t R = static_cast<size_t>(n), RK = R * K;
  NH_PF_TRY(DevAllocN(&h, R * d));
  NH_PF_TRY(DevAllocN(&q, R * d));
  NH_PF_TRY(DevAllocN(&k, R * dkv));
  NH_PF_TRY(DevAllocN(&v, R * dkv));
  NH_PF_TRY(DevAllocN(&qr, R * d));
  NH_PF_TRY(DevAllocN(&att, R * d));
  NH_PF_TRY(DevAllocN(&xn, R * d));
  NH_PF_TRY(DevAllocN(&wts, RK));
  NH_PF_TRY(DevAllocN(&ff, RK * F));
  NH_PF_TRY(DevAllocN(&y, RK * d));
  NH_PF_TRY(DevAllocN(&q8, static_cast<size_t>(nh_batch_q8_bytes(n, c.n_embd))));
  NH_PF_TRY(DevAllocN(&q8ff, static_cast<size_t>(nh_batch_q8_bytes(static_cast<int64_t>(RK), c.n_ff))));
  NH_PF_TRY(DevAllocN(&sel, RK));
  NH_PF_TRY(DevAllocN(&off, c.n_expert));
  NH_PF_TRY(DevAllocN(&cnt, c.n_expert));
  NH_PF_TRY(DevAllocN(&act_idx, RK));
  NH_PF_TRY(DevAllocN(&out_idx, RK));
  rows = n;
  return NH_OK;
}

bool Engine::PrefillSupported(const ModelView& m, bool experts_resident) {
  const OlmoeConfig& c = m.cfg;
  const int64_t hd = c.head_dim();
  if (!RowLenOk(c.n_embd) || !RowLenOk(c.n_ff) || hd % 32 != 0 || hd > 128 || c.n_expert == 0 ||
      c.n_expert > 256 || c.n_expert_used == 0 || c.n_expert_used > 32 || c.n_embd % 4 != 0)
    return false;
  if (!QuantType(m.te) && m.te != NH_TYPE_F32) return false;
  for (const LayerView& L : m.layers) {
    for (int32_t t : {L.tq, L.tk, L.tv, L.to})
      if (!QuantType(t)) return false;
    if (!experts_resident) continue;  // streamed experts: the slot pools' products take any row count
    for (int32_t t : {L.tg, L.tu, L.td})
      if (!QuantType(t)) return false;
    if (L.gate == nullptr || L.up == nullptr || L.down == nullptr) return false;
  }
  return true;
}

int Engine::Prefill(const ModelView& m, int n_tok, bool norm_topk, bool trace) {
  if (n_tok <= 0) return NH_OK;
  if (!PrefillSupported(m)) return NH_E_TYPE;
  if (n_tok >= max_seq_) return NH_E_CAPACITY;
  const OlmoeConfig& c = cfg_;
  if (!pf_) pf_.reset(new PrefillBuffers());
  NH_PF_TRY(pf_->Reserve(c, std::min(n_tok, kPrefillChunk)));
  PrefillBuffers& b = *pf_;
  const int64_t d = c.n_embd, hd = c.head_dim(), dkv = static_cast<int64_t>(c.n_head_kv) * hd, F = c.n_ff;
  const int E = static_cast<int>(c.n_expert), K = static_cast<int>(c.n_expert_used), L = static_cast<int>(c.n_layers);
  const float eps = c.rms_eps;
  const float kq_scale = 1.0f / std::sqrt(static_cast<float>(hd));
  cudaStream_t s = stream_;
  for (int p0 = 0; p0 < n_tok; p0 += kPrefillChunk) {
    const int T = std::min(kPrefillChunk, n_tok - p0);
    auto dense = [&](const void* w, int32_t type, int64_t rows, const void* act, float* out, int64_t stride,
                     int mode) {
      NhGroupedRowDot g;
      std::memset(&g, 0, sizeof(g));
      g.w = w;
      g.type = type;
      g.type2 = type;
      g.n = d;
      g.rows = rows;
      g.n_groups = 1;
      g.n_tok = T;
      g.max_tokens = T;
      g.q8 = act;
      g.out = out;
      g.out_stride = stride;
      g.mode = mode;
      g.err = &state_->error;
      return nh_batch_rowdot(&g, s);
    };
    NH_PF_TRY(nh_prefill_embed(prompt_ + p0, T, m.embd, m.te, d, c.n_vocab, b.h, &state_->error, s));
    for (int l = 0; l < L; ++l) {
      const LayerView& Lv = m.layers[l];
      // Attention block (attention.cc:79-134).
      NH_PF_TRY(nh_batch_prep(b.h, d, T, Lv.attn_norm, eps, 1, d, b.q8, nullptr, s));
      NH_PF_TRY(dense(Lv.wq, Lv.tq, d, b.q8, b.q, d, NH_ROWDOT_STORE));
      NH_PF_TRY(dense(Lv.wk, Lv.tk, dkv, b.q8, b.k, dkv, NH_ROWDOT_STORE));
      NH_PF_TRY(dense(Lv.wv, Lv.tv, dkv, b.q8, b.v, dkv, NH_ROWDOT_STORE));
      NH_PF_TRY(nh_prefill_qk(b.q, b.k, b.v, Lv.q_norm, Lv.k_norm, eps, T, p0, c.n_head, c.n_head_kv,
                              static_cast<int>(hd), rope_cs_, kv_->k(l), kv_->v(l), max_seq_, b.qr, s));
      NH_PF_TRY(nh_prefill_attention(b.qr, T, p0, c.n_head, c.n_head_kv, static_cast<int>(hd), kq_scale, kv_->k(l),
                                     kv_->v(l), max_seq_, b.att, s));
      NH_PF_TRY(nh_batch_prep(b.att, d, T, nullptr, eps, 0, d, b.q8, nullptr, s));
      NH_PF_TRY(dense(Lv.wo, Lv.to, d, b.q8, b.h, d, NH_ROWDOT_RESIDUAL));
      // MoE block (moe.cc:7-63).
      NH_PF_TRY(nh_batch_prep(b.h, d, T, Lv.ffn_norm, eps, 1, d, b.q8, b.xn, s));
      NH_PF_TRY(nh_batch_router_trace(b.xn, Lv.router, T, d, E, K, norm_topk ? 1 : 0, b.sel, b.wts,
                                      trace ? trace_sel_ : nullptr, trace ? trace_gap_ : nullptr, p0, l, L, s));
      NH_PF_TRY(nh_batch_moe_plan(b.sel, T, K, E, b.off, b.cnt, b.act_idx, b.out_idx, s));
      NhGroupedRowDot g;
      std::memset(&g, 0, sizeof(g));
      g.w = Lv.gate;
      g.w2 = Lv.up;
      g.mstride = Lv.gate_nb2;
      g.mstride2 = Lv.up_nb2;
      g.type = Lv.tg;
      g.type2 = Lv.tu;
      g.n = d;
      g.rows = F;
      g.n_groups = E;
      g.off = b.off;
      g.cnt = b.cnt;
      g.act_idx = b.act_idx;
      g.out_idx = b.out_idx;
      g.max_tokens = T;
      g.q8 = b.q8;
      g.out = b.ff;
      g.out_stride = F;
      g.mode = NH_ROWDOT_SWIGLU;
      g.err = &state_->error;
      NH_PF_TRY(nh_batch_rowdot(&g, s));
      NH_PF_TRY(nh_batch_prep(b.ff, F, static_cast<int64_t>(T) * K, nullptr, eps, 0, F, b.q8ff, nullptr, s));
      std::memset(&g, 0, sizeof(g));
      g.w = Lv.down;
      g.mstride = Lv.down_nb2;
      g.type = Lv.td;
      g.type2 = Lv.td;
      g.n = F;
      g.rows = d;
      g.n_groups = E;
      g.off = b.off;
      g.cnt = b.cnt;
      g.act_idx = b.out_idx;  // the ff row of pair j is its (token, slot) index
      g.out_idx = b.out_idx;
      g.max_tokens = T;
      g.q8 = b.q8ff;
      g.out = b.y;
      g.out_stride = d;
      g.mode = NH_ROWDOT_STORE;
      g.err = &state_->error;
      NH_PF_TRY(nh_batch_rowdot(&g, s));
      NH_PF_TRY(nh_batch_combine(b.y, b.wts, T, K, d, b.h, s));
    }
  }
  return NH_OK;
}

}  // namespace nuthatch

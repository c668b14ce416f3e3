/* nh_kernels.h — C ABI of the sm_100a kernels behind nuthatch's per-token
 * OLMoE forward.
 *
 * Every entry point launches on `stream` (a cudaStream_t passed as void*),
 * never synchronises and never allocates.  Device buffers are owned by the
 * caller.  Return value: NH_OK or a negative NH_E_* code (argument checks are
 * done on the host before any launch).  Citations name the reference call
 * site (file:line within chen3feng/nuthatch) each kernel replaces; the
 * reference runs those ops on ggml's CPU backend.
 *
 * Weights stay in their native GGUF super-block layout (Q4_K: 144 bytes per
 * 256 values, Q6_K: 210 bytes per 256 values, or F32).  Device regions that
 * hold weights must carry at least 32 bytes of readable tail padding: rows are
 * staged with 16-byte copies rounded outwards.
 *
 * Kernels taking an NhDecodeState* record a failed bounded device-side wait
 * as NH_E_TIMEOUT in state->error (the state may be NULL for the standalone
 * forms, which then only stop early).
 *
 * Activations that meet a quantised weight are quantised to Q8_K inside the
 * kernel exactly as ggml's CPU mul_mat does (per 256 values: the element of
 * largest magnitude maps to -127, round half to even), and each 256-value
 * super-block contributes an exact integer dot product scaled in f32.
 */
#ifndef NH_KERNELS_H_
#define NH_KERNELS_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NH_TYPE_F32 0
#define NH_TYPE_Q4_K 12
#define NH_TYPE_Q6_K 14

#define NH_OK 0
#define NH_E_ARG (-1)         /* bad argument (null pointer, size, unsupported shape) */
#define NH_E_CUDA (-2)        /* a CUDA launch or API call failed */
#define NH_E_TYPE (-3)        /* unsupported tensor type for this kernel */
#define NH_E_IO (-4)          /* file or read error (host API) */
#define NH_E_STATE (-5)       /* object in the wrong state (host API) */
#define NH_E_NOMEM (-6)       /* device or host allocation failed (host API) */
#define NH_E_CAPACITY (-7)    /* request beyond a stated capacity */
#define NH_E_TIMEOUT (-8)     /* a bounded device-side wait expired (recorded in NhDecodeState.error) */

/* Per-sequence decode cursor, resident in device memory.  The kernels read
 * `pos` (tokens already in the KV cache); nh_lm_head_argmax advances it, so a
 * captured step can be replayed without the host.  Token ids for positions
 * below n_prompt come from the prompt array; later ones from `token`, the id
 * the last argmax fed back (generate.cc:93-102). */
typedef struct NhDecodeState {
  int32_t pos;
  int32_t n_prompt;
  int32_t n_predict;
  int32_t n_out;   /* generated ids written so far */
  int32_t token;   /* id fed back by the last argmax */
  int32_t error;   /* first kernel-side error code, 0 if none */
  int32_t pad0;
  int32_t pad1;
} NhDecodeState;

/* Query helpers. */
int nh_device_sm_count(int device);
/* Bytes of scratch the split attention / argmax reductions need; see the
 * kernels below. */
int64_t nh_attention_scratch_bytes(int n_head, int head_dim, int max_seq);
int64_t nh_argmax_scratch_bytes(int n_vocab);

/* The k selected expert ids of a router step handed to the host without a
 * stream synchronisation (no reference counterpart: the two-phase streaming
 * form's selection read-back, streaming_forward.cc:228-236): copies sel[0..k)
 * to host_sel and then writes seq to *host_seq, both in mapped pinned host
 * memory (device addresses from cudaHostGetDevicePointer), with a
 * system-scope fence between; the host waits until *host_seq == seq.  k <= 32. */
int nh_publish_selection(const int32_t* sel, int k, int32_t* host_sel, uint32_t* host_seq, uint32_t seq,
                         void* stream);

/* Embedding row lookup for the token at state->pos (ggml_get_rows on
 * token_embd, forward.cc:53-54, streaming_forward.cc:58-66): dequantises one
 * row of `table` ([n_vocab] rows of n_embd) into h_out. */
int nh_embed_step(const NhDecodeState* state, const int32_t* prompt_ids, const void* table,
                  int32_t type, int64_t n_embd, int64_t n_vocab, float* h_out, void* stream);

/* RMSNorm(h)*attn_norm followed by the Q, K and V projections
 * (attention.cc:79-83): q_out[n_embd], k_out[n_embd_kv], v_out[n_embd_kv].
 * Each weight may be F32, Q4_K or Q6_K independently. */
int nh_qkv_proj(NhDecodeState* state, const float* h, const float* attn_norm, float eps, const void* wq,
                int32_t tq, const void* wk, int32_t tk, const void* wv, int32_t tv, int64_t n_embd,
                int64_t n_embd_kv, float* q_out, float* k_out, float* v_out, void* stream);

/* One decode position of cached attention (attention.cc:84-133): QK-norm
 * over the full width (q_norm over n_embd, k_norm over n_embd_kv), NEOX RoPE
 * at state->pos, append post-RoPE K and raw V to the f32 caches
 * ([max_seq][n_embd_kv] per layer, kv_cache.cc:11-22), then causal softmax
 * attention over positions 0..pos split across CTAs with a deterministic
 * combine.  rope_cs is a [max_seq][head_dim/2] table of (cos, sin) pairs for
 * theta_i = pos * base^(-2i/head_dim), theta advanced by repeated f32
 * multiplication as ggml_rope_ext does (attention.cc:88-93); nh_rope_table
 * fills it.  kq_scale = 1/sqrtf(head_dim) (attention.cc:126).  `scratch`
 * holds nh_attention_scratch_bytes() bytes, zeroed once before first use (the
 * kernel leaves its counters zeroed). */
int nh_attention_step(const NhDecodeState* state, const float* q, const float* k,
                      const float* v, const float* q_norm, const float* k_norm, float eps,
                      int n_head, int n_head_kv, int head_dim, const float* rope_cs,
                      float kq_scale, float* k_cache, float* v_cache, int max_seq,
                      void* scratch, float* attn_out, void* stream);

/* No counterpart in the reference.  nh_attention_step without the caller's
 * scratch buffer, for callers that cannot allocate device memory: code that
 * runs inside an allocator hook or memory-pool callback (calling the
 * allocator there would re-enter it), plugin hosts that own every device
 * allocation, and processes whose allocator is already at its limit.  The
 * split-combine scratch is a static device array of
 * NH_ATTN_STATIC_SCRATCH_BYTES that each GPU loading the library holds until
 * the process exits; nothing is allocated per call.  Same arguments and
 * results as nh_attention_step minus `scratch`.
 *   - Returns NH_E_CAPACITY, launching nothing, when
 *     nh_attention_scratch_bytes(n_head, head_dim, max_seq) exceeds
 *     NH_ATTN_STATIC_SCRATCH_BYTES or n_head > 64 (for head_dim 128 and 16
 *     heads that allows max_seq up to 7,936).
 *   - Every argument check runs first: a rejected call enqueues nothing.
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *     The address is kept for the life of the process; after cudaDeviceReset
 *     on a device it is stale, so do not call this entry there again.
 *   - Every call clears the array's split counters on `stream`, then runs the
 *     step there.  All calls on a device share its one array and it keeps the
 *     last call's contents: calls that can overlap on the GPU (issued to
 *     streams with no ordering between them) race on it, so the caller must
 *     serialise them. */
#define NH_ATTN_STATIC_SCRATCH_BYTES (1 << 20)
int nh_attention_step_static(const NhDecodeState* state, const float* q, const float* k,
                             const float* v, const float* q_norm, const float* k_norm, float eps,
                             int n_head, int n_head_kv, int head_dim, const float* rope_cs,
                             float kq_scale, float* k_cache, float* v_cache, int max_seq,
                             float* attn_out, void* stream);

/* Host helper: fills rope_cs_host[max_seq][head_dim/2][2] (see above). */
void nh_rope_table(float base, int head_dim, int max_seq, float* rope_cs_host);

/* h_io[r] = h_io[r] + (W . x)[r]: output projection plus residual
 * (attention.cc:134, forward.cc:65-67). */
int nh_out_proj_residual(NhDecodeState* state, const float* x, const void* wo, int32_t to,
                         int64_t n_embd, float* h_io, void* stream);

/* Router (moe.cc:16-37, streaming_forward.cc:101-117): RMSNorm(h)*ffn_norm,
 * F32 router GEMV, softmax over n_expert, top-k in descending probability
 * (equal probabilities: lower expert id first), the selected probabilities
 * (renormalised when norm_topk, clamped sum 6.103515625e-5).  Writes sel[k],
 * wts[k]; when trace_sel is not null also trace_sel[pos*n_layers*k + layer*k
 * + i] and trace_gap[pos*n_layers + layer] (the smallest difference between
 * adjacent probabilities of the descending top-(k+1): the near-tie measure). */
int nh_router_topk(const NhDecodeState* state, const float* h, const float* ffn_norm,
                   float eps, const float* router, int64_t n_embd, int n_expert, int k,
                   int norm_topk, int32_t* sel, float* wts, int32_t* trace_sel,
                   float* trace_gap, int layer, int n_layers, void* scratch, void* stream);
int64_t nh_router_scratch_bytes(int n_expert);


/* Expert up/gate projections and SwiGLU (moe.cc:41-46): for i < k,
 * ff[i][r] = silu((gate_e . b)[r]) * (up_e . b)[r] with e = wsel[i] and
 * b = RMSNorm(h)*ffn_norm.  gate/up are [n_slots][n_ff][n_embd] with
 * per-expert stride *_nb2 bytes (the resident expert tensors or the slot pool). */
int nh_moe_gate_up(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                   const int32_t* wsel, int k,
                   const void* gate, int32_t tg, uint64_t gate_nb2, const void* up, int32_t tu,
                   uint64_t up_nb2, int64_t n_embd, int64_t n_ff, float* ff, void* stream);
/* nh_moe_gate_up that also starts the selected experts' down slices
 * (down + wsel[i] * down_nb2, down_nb2 bytes each) towards L2, each CTA a
 * share, so nh_moe_down_combine reads them from L2.  A performance hint only:
 * results are those of nh_moe_gate_up; down may be null. */
int nh_moe_gate_up_prefetch(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                            const int32_t* wsel, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                            const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff,
                            float* ff, const void* down, uint64_t down_nb2, void* stream);

/* Down projections, routing weights and residual (moe.cc:47-60,
 * forward.cc:76-78): h_io[r] = h_io[r] + sum_i wts[i]*(down_e . ff[i])[r],
 * the products rounded before the adds and summed in top-k order.  When
 * dump is not null and state->pos >= n_prompt-1, h_io is also copied to
 * dump[(pos-n_prompt+1)*dump_step_stride + dump_offset + r]. */
int nh_moe_down_combine(const NhDecodeState* state, const float* ff, const int32_t* wsel,
                        const float* wts, int k, const void* down, int32_t td,
                        uint64_t down_nb2, int64_t n_ff, int64_t n_embd, float* h_io,
                        float* dump, int64_t dump_step_stride, int64_t dump_offset,
                        void* stream);

/* nh_moe_gate_up_prefetch and nh_moe_down_combine with the k selected slots
 * given in HOST memory (slots[0..k), read during the call and passed with the
 * launch), for the streaming form whose host decides the slots: no copy of
 * the selection has to reach the device before the kernels run. */
int nh_moe_gate_up_slots(NhDecodeState* state, const float* h, const float* ffn_norm, float eps,
                         const int32_t* slots, int k, const void* gate, int32_t tg, uint64_t gate_nb2,
                         const void* up, int32_t tu, uint64_t up_nb2, int64_t n_embd, int64_t n_ff,
                         float* ff, const void* down, uint64_t down_nb2, void* stream);
int nh_moe_down_combine_slots(const NhDecodeState* state, const float* ff, const int32_t* slots,
                              const float* wts, int k, const void* down, int32_t td, uint64_t down_nb2,
                              int64_t n_ff, int64_t n_embd, float* h_io, float* dump,
                              int64_t dump_step_stride, int64_t dump_offset, void* stream);

/* The whole MoE block of one layer (moe.cc:16-60, forward.cc:69-78) as one
 * cooperative kernel: nh_router_topk, nh_moe_gate_up and nh_moe_down_combine
 * in sequence, the same results bit for bit, with the stages separated by
 * device-side waits instead of kernel boundaries.  Q4_K/Q6_K expert tensors
 * with n_embd/256 and n_ff/256 in {1,2,4,8} and (32/(n_ff/256)) % k == 0;
 * outside that range (or when the grid cannot be co-resident) it returns
 * NH_E_ARG or NH_E_TYPE having launched nothing, and the three kernels above
 * do the work.  `scratch`: nh_moe_layer_scratch_bytes(n_expert) bytes,
 * zeroed once before the first call.  Between calls it keeps a launch count
 * and the router logits tagged with it, so keep using the same (unmodified)
 * scratch, or zero it again, and give calls that may overlap on the GPU
 * separate scratch. */
typedef struct NhMoeLayer {
  NhDecodeState* state;
  float* h;                 /* in: the residual stream; out: h + MoE(h) */
  const float* ffn_norm;
  float eps;
  const float* router;      /* [n_expert][n_embd] f32 */
  int64_t n_embd, n_ff;
  int n_expert, k, norm_topk, layer, n_layers;
  const void* gate;
  int32_t tg;
  uint64_t gate_nb2;
  const void* up;
  int32_t tu;
  uint64_t up_nb2;
  const void* down;
  int32_t td;
  uint64_t down_nb2;
  int32_t* sel;             /* [k] selected experts (router output) */
  float* wts;               /* [k] their weights */
  int32_t* trace_sel;       /* optional, as nh_router_topk */
  float* trace_gap;
  float* ff;                /* [k][n_ff] */
  float* dump;              /* optional, as nh_moe_down_combine */
  int64_t dump_step_stride, dump_offset;
  void* scratch;
} NhMoeLayer;
int64_t nh_moe_layer_scratch_bytes(int n_expert);
int nh_moe_layer(const NhMoeLayer* layer, void* stream);


/* Output norm, lm_head GEMV and greedy argmax (forward.cc:81-83,
 * generate.cc:93-102): first maximum wins.  Skipped (beyond the state
 * advance) for positions before the last prompt token.  The last CTA writes
 * out_tokens[n_out], feeds the id back into state->token, and advances
 * state->pos (and n_out).  logits_dump, when not null, receives the logits of
 * each generated step at [(pos-n_prompt+1)*n_vocab]. */
int nh_lm_head_argmax(NhDecodeState* state, const float* h, const float* out_norm, float eps,
                      const void* w, int32_t tw, int64_t n_embd, int64_t n_vocab,
                      int32_t* out_tokens, float* logits_dump, void* scratch, void* stream);

/* ---- batched decode: B sequences advanced one position per step in lockstep
 * (the batched form of GreedyGenerateCached, generate.cc:55-106, for
 * independent sequences of equal prompt length).  The shared cursor
 * NhDecodeState.pos is the position every sequence is at.  Per token the
 * arithmetic equals the batch-1 kernels', so each sequence's ids equal a
 * batch-1 decode of it.  Q8 activation rows are K/256 blocks of 304 bytes
 * (int8 quants[256] in element order, int16 sums[16], f32 scale, padding). */

/* Bytes of a Q8 activation buffer of `rows` rows of n values. */
int64_t nh_batch_q8_bytes(int64_t rows, int64_t n);

/* h[b] = embedding row of sequence b's token at state->pos (prompts
 * [n_seq][n_prompt], later the fed-back id fed[b]). */
int nh_batch_embed(const NhDecodeState* state, const int32_t* prompts, int n_prompt, const int32_t* fed,
                   int n_seq, const void* table, int32_t type, int64_t n_embd, int64_t n_vocab, float* h,
                   void* stream);

/* Per row r < rows of x (row stride x_stride floats): optional RMSNorm * norm_w
 * (do_norm), then Q8_K into q8 (may be null) and the normalised f32 row into
 * xn (may be null; [rows][n]). */
int nh_batch_prep(const float* x, int64_t x_stride, int64_t rows, const float* norm_w, float eps, int do_norm,
                  int64_t n, void* q8, float* xn, void* stream);

#define NH_ROWDOT_STORE 0    /* out[o][row] = W.x */
#define NH_ROWDOT_RESIDUAL 1 /* out[o][row] += W.x */
#define NH_ROWDOT_SWIGLU 2   /* out[o][row] = silu(W.x) * (W2.x) */

/* Grouped row dots over Q4_K/Q6_K matrices of n <= 2048 columns (ggml_mul_mat
 * and, with groups, mul_mat_id, moe.cc:41-50).  Group e multiplies matrix
 * w + e*mstride (rows x n) with tokens j in [off[e], off[e]+cnt[e]): token j
 * reads Q8 row act_idx[j] and writes output row out_idx[j].  With off null
 * there is one group over tokens 0..n_tok-1 (identity indices).  max_tokens
 * bounds any group's token count. */
typedef struct NhGroupedRowDot {
  const void* w;
  const void* w2;
  uint64_t mstride, mstride2;
  int32_t type, type2;
  int64_t n, rows;
  int32_t n_groups;
  const int32_t* off;
  const int32_t* cnt;
  const int32_t* act_idx;
  const int32_t* out_idx;
  int32_t n_tok, max_tokens;
  const void* q8;
  float* out;
  int64_t out_stride;
  int32_t mode;
  int32_t engine;  /* NH_ROWDOT_ENGINE_*: which implementation (all give identical results) */
  int32_t* err;    /* optional: NH_E_TIMEOUT is recorded here if a bounded device wait expires */
} NhGroupedRowDot;
#define NH_ROWDOT_ENGINE_AUTO 0  /* tensor cores (tcgen05) for Q4_K at >= 128 tokens, else mma.sync */
#define NH_ROWDOT_ENGINE_DP4A 1  /* CUDA-core integer dots */
#define NH_ROWDOT_ENGINE_MMA 2   /* mma.sync m16n8k32 / m16n8k16 int8, accumulators in registers */
#define NH_ROWDOT_ENGINE_TC 3    /* tcgen05.mma kind::i8, accumulators in tensor memory (Q4_K only) */
int nh_batch_rowdot(const NhGroupedRowDot* g, void* stream);

/* The tcgen05 form directly (ggml_mul_mat_id on the 5th-generation tensor
 * cores): Q4_K weights (both matrices for SwiGLU), n a power-of-two multiple
 * of 256 up to 2048, 16-byte aligned weights, strides and Q8 rows.  One 32-value
 * sub-block per kind::i8 MMA into its own tensor-memory accumulator, scales
 * applied in registers in the row-dot order: results identical to the other
 * engines.  NH_E_TYPE / NH_E_ARG (nothing launched) outside that.  A CTA owns
 * 128 rows x 32 tokens of one group; grid (groups x row tiles, max_tokens/32). */
int nh_batch_rowdot_tc(const NhGroupedRowDot* g, void* stream);
/* 1 unless the environment sets NH_TC=0 (read once): whether
 * NH_ROWDOT_ENGINE_AUTO may pick the tensor-core form. */
int nh_tc_enabled(void);

/* Per sequence: QK-norm over the full q/k width, NEOX RoPE at state->pos,
 * rotated q into qr [n_seq][n_head*head_dim], and the new K/V rows appended to
 * the caches ([n_seq][max_seq][n_head_kv*head_dim] per layer). */
int nh_batch_qk(const NhDecodeState* state, const float* q, const float* k, const float* v, const float* q_norm,
                const float* k_norm, float eps, int n_seq, int n_head, int n_head_kv, int head_dim,
                const float* rope_cs, float* k_cache, float* v_cache, int max_seq, float* qr, void* stream);

/* Attention of every sequence over positions 0..state->pos in 64-position
 * splits combined in order (the batch-1 kernel's arithmetic).  `scratch`:
 * nh_batch_attention_scratch_bytes() bytes, zeroed once. */
int64_t nh_batch_attention_scratch_bytes(int n_seq, int n_head, int head_dim, int max_seq);
int nh_batch_attention(const NhDecodeState* state, const float* qr, int n_seq, int n_head, int n_head_kv,
                       int head_dim, float kq_scale, const float* k_cache, const float* v_cache, int max_seq,
                       void* scratch, float* out, void* stream);

/* Router per token from the normalised rows xn [n_seq][n_embd]: sel/wts
 * [n_seq][k] as nh_router_topk. */
int nh_batch_router(const float* xn, const float* router, int n_seq, int64_t n_embd, int n_expert, int k,
                    int norm_topk, int32_t* sel, float* wts, void* stream);

/* nh_batch_router that also records row b as the routing of position
 * trace_pos0 + b in layer `layer` (trace_sel[((trace_pos0+b)*n_layers +
 * layer)*k + i], trace_gap[(trace_pos0+b)*n_layers + layer], the layout of
 * nh_router_topk's trace; both may be null). */
int nh_batch_router_trace(const float* xn, const float* router, int n_seq, int64_t n_embd, int n_expert, int k,
                          int norm_topk, int32_t* sel, float* wts, int32_t* trace_sel, float* trace_gap,
                          int trace_pos0, int layer, int n_layers, void* stream);

/* Per-expert token lists of sel [n_seq][k] in (token, slot) order: off/cnt
 * [n_expert], act_idx[j] = token, out_idx[j] = token*k + slot. */
int nh_batch_moe_plan(const int32_t* sel, int n_seq, int k, int n_expert, int32_t* off, int32_t* cnt,
                      int32_t* act_idx, int32_t* out_idx, void* stream);

/* nh_batch_moe_plan over experts [e_first, e_first + n_expert) only (group
 * e - e_first); pairs that selected other experts are left out.  Expert
 * parallelism plans a rank's own shard over every rank's tokens with it. */
int nh_batch_moe_plan_range(const int32_t* sel, int n_seq, int k, int e_first, int n_expert, int32_t* off,
                            int32_t* cnt, int32_t* act_idx, int32_t* out_idx, void* stream);

/* Expert-parallel combine (moe.cc:51-60 on the token's home GPU): h[b] +=
 * sum_i wts[b][i] * row(b, i), products rounded, in top-k order, where
 * row(b, i) is row b*k+i of block sel[b][i] / experts_per_rank of y_recv
 * (n_src blocks of src_stride floats: the pick rows each expert-owning rank
 * returned). */
int nh_ep_combine(const float* y_recv, int64_t src_stride, int n_src, const int32_t* sel, const float* wts, int n_seq,
                  int k, int64_t n_embd, int experts_per_rank, float* h, void* stream);

/* h[b] += sum_i wts[b][i] * y[b*k+i] (products rounded, top-k order). */
int nh_batch_combine(const float* y, const float* wts, int n_seq, int k, int64_t n_embd, float* h, void* stream);

/* Greedy ids from logits [n_seq][n_vocab] (first maximum); from the last
 * prompt position on writes out_tokens[b][pos-n_prompt+1] and fed[b]; the
 * last CTA advances state->pos.  scratch: 64 zeroed bytes. */
int nh_batch_argmax(NhDecodeState* state, const float* logits, int n_seq, int64_t n_vocab, int32_t* fed,
                    int32_t* out_tokens, int n_predict, void* scratch, void* stream);

/* ---- prompt prefill: the n_tok positions pos0 .. pos0+n_tok-1 of ONE
 * sequence as rows of the batched kernels (the reference forwards the whole
 * prompt in its first GreedyGenerateCached step, generate.cc:63-91;
 * forward.cc:45-79).  Per position the arithmetic equals the batch-1
 * kernels', so the K/V rows and ids that follow are identical to a
 * position-by-position prompt.  The caches are one sequence's
 * [max_seq][n_head_kv*head_dim] per layer. */

/* h[r] = embedding row of ids[r] (ggml_get_rows, forward.cc:53-54); an id
 * outside the vocabulary reads row 0 and sets *err to NH_E_ARG (err may be
 * null). */
int nh_prefill_embed(const int32_t* ids, int n_tok, const void* table, int32_t type, int64_t n_embd,
                     int64_t n_vocab, float* h, int32_t* err, void* stream);

/* nh_batch_qk for prefill rows: row r is at position pos0 + r; QK-norm, NEOX
 * RoPE and the K/V append at that position (attention.cc:84-116). */
int nh_prefill_qk(const float* q, const float* k, const float* v, const float* q_norm, const float* k_norm, float eps,
                  int n_tok, int pos0, int n_head, int n_head_kv, int head_dim, const float* rope_cs,
                  float* k_cache, float* v_cache, int max_seq, float* qr, void* stream);

/* Causal attention of the prefill rows (attention.cc:119-133 with the mask
 * offset n_past = pos0): row r attends cache positions 0..pos0+r, in the
 * 64-position splits of nh_attention_step combined in the same order.
 * head_dim a multiple of 32, at most 128; caches and qr 16-byte aligned. */
int nh_prefill_attention(const float* qr, int n_tok, int pos0, int n_head, int n_head_kv, int head_dim,
                         float kq_scale, const float* k_cache, const float* v_cache, int max_seq, float* out,
                         void* stream);

/* The same three over n_seq sequences in one launch each, every sequence
 * contributing n_tok rows at positions pos0..pos0+n_tok-1 (row r is
 * sequence r / n_tok): ids of sequence s at ids + s*ids_stride; q, k, v, qr
 * and out [n_seq*n_tok][...]; caches [n_seq][max_seq][n_head_kv*head_dim]. */
int nh_prefill_embed_seqs(const int32_t* ids, int64_t ids_stride, int n_seq, int n_tok, const void* table,
                          int32_t type, int64_t n_embd, int64_t n_vocab, float* h, int32_t* err, void* stream);
int nh_prefill_qk_seqs(const float* q, const float* k, const float* v, const float* q_norm, const float* k_norm,
                       float eps, int n_seq, int n_tok, int pos0, int n_head, int n_head_kv, int head_dim,
                       const float* rope_cs, float* k_cache, float* v_cache, int max_seq, float* qr, void* stream);
int nh_prefill_attention_seqs(const float* qr, int n_seq, int n_tok, int pos0, int n_head, int n_head_kv,
                              int head_dim, float kq_scale, const float* k_cache, const float* v_cache, int max_seq,
                              float* out, void* stream);

/* ---- standalone forms used by the parity tests ---- */

/* y[r] = (W . x)[r] for r < rows (ggml_mul_mat for one activation row); when
 * norm_w is not null x is first RMS-normalised and multiplied by norm_w. */
int nh_gemv(NhDecodeState* state, const void* w, int32_t type, int64_t n, int64_t rows,
            const float* x, const float* norm_w, float eps, float* y, void* stream);

/* Q8_K quantisation of n values (n a multiple of 256) into 292-byte blocks
 * (f32 d, int8 qs[256], int16 bsums[16]). */
int nh_quantize_q8k(const float* x, int64_t n, void* out, void* stream);

/* y[i] = exp(x[i]) as the kernels compute it (Cody-Waite reduction, degree-7
 * Taylor polynomial, IEEE f32 steps); used by softmax and SiLU. */
int nh_exp_cw(const float* x, int64_t n, float* y, void* stream);

/* Dequantise `rows` rows of n values (ggml dequantize_row_*). */
int nh_dequantize(const void* w, int32_t type, int64_t n, int64_t rows, float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NH_KERNELS_H_ */

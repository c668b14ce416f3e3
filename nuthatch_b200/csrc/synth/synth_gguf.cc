// Seeded synthetic OLMoE-shaped GGUF writer.
//
// Produces GGUF v3 files with the tensor names, shapes and metadata keys that
// the reference loader reads (olmoe_model.cc:31-54 for the keys,
// forward.cc:14-42 and moe.cc:7-63 for the tensor names).  Weights are drawn
// from an approximately normal distribution (Irwin-Hall sum of four uniforms,
// rescaled to unit variance, times `weight_std`) by a counter-based hash, so
// the bytes of a file depend only on the spec and never on the thread count.
// 1-D norm weights are 1.0 (F32).  The router (`ffn_gate_inp`) stays F32.
//
// Quantisation mode 1 is a Q4_K_M-like mix: Q4_K everywhere, except attn_v and
// ffn_down on odd layers and `output`, which are Q6_K.  Any tensor whose row
// length is not a multiple of 256 falls back to F32.
//
// The quantisers here are this project's own simple min/max schemes; they only
// have to produce valid Q4_K / Q6_K super-blocks (144 / 210 bytes per 256
// values) in the GGUF layout that gguf-py's dequantisers read.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr int kQK = 256;
constexpr uint32_t kTypeF32 = 0;
constexpr uint32_t kTypeQ4K = 12;
constexpr uint32_t kTypeQ6K = 14;
constexpr size_t kQ4KBytes = 144;
constexpr size_t kQ6KBytes = 210;
constexpr size_t kAlign = 32;

uint64_t Mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

uint64_t HashName(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) h = (h ^ c) * 1099511628211ull;
  return h;
}

// Irwin-Hall(4) normal approximation with unit variance, from one 64-bit hash.
inline float NormalApprox(uint64_t key) {
  const uint64_t h = Mix64(key);
  float s = 0.f;
  for (int i = 0; i < 4; ++i) {
    s += (static_cast<float>((h >> (16 * i)) & 0xFFFF) + 0.5f) * (1.0f / 65536.0f);
  }
  return (s - 2.0f) * 1.7320508f;
}

inline uint16_t ToHalf(float f) {
  _Float16 h = static_cast<_Float16>(f);
  uint16_t u;
  std::memcpy(&u, &h, 2);
  return u;
}
inline float FromHalf(uint16_t u) {
  _Float16 h;
  std::memcpy(&h, &u, 2);
  return static_cast<float>(h);
}

inline int RoundClamp(float v, int lo, int hi) {
  int q = static_cast<int>(std::lrintf(v));
  return std::min(hi, std::max(lo, q));
}

// One Q4_K super-block: value = d*sc[j]*q - dmin*m[j], q in 0..15, 8 sub-blocks of 32.
void QuantizeQ4K(const float* x, uint8_t* out) {
  float scale[8], mins[8];
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int i = 1; i < 32; ++i) {
      mn = std::min(mn, x[32 * j + i]);
      mx = std::max(mx, x[32 * j + i]);
    }
    mn = std::min(mn, 0.f);
    scale[j] = (mx - mn) / 15.f;
    mins[j] = -mn;
  }
  float smax = 0.f, mmax = 0.f;
  for (int j = 0; j < 8; ++j) {
    smax = std::max(smax, scale[j]);
    mmax = std::max(mmax, mins[j]);
  }
  const uint16_t dh = ToHalf(smax / 63.f);
  const uint16_t mh = ToHalf(mmax / 63.f);
  const float d = FromHalf(dh), dmin = FromHalf(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d > 0 ? RoundClamp(scale[j] / d, 0, 63) : 0;
    m[j] = dmin > 0 ? RoundClamp(mins[j] / dmin, 0, 63) : 0;
  }
  int q[kQK];
  for (int j = 0; j < 8; ++j) {
    const float step = d * sc[j];
    const float off = dmin * m[j];
    for (int i = 0; i < 32; ++i) {
      q[32 * j + i] = step > 0 ? RoundClamp((x[32 * j + i] + off) / step, 0, 15) : 0;
    }
  }
  std::memcpy(out + 0, &dh, 2);
  std::memcpy(out + 2, &mh, 2);
  uint8_t* s = out + 4;
  for (int i = 0; i < 4; ++i) {
    s[i] = static_cast<uint8_t>((sc[i] & 63) | ((sc[4 + i] >> 4) << 6));
    s[4 + i] = static_cast<uint8_t>((m[i] & 63) | ((m[4 + i] >> 4) << 6));
    s[8 + i] = static_cast<uint8_t>((sc[4 + i] & 15) | ((m[4 + i] & 15) << 4));
  }
  uint8_t* qs = out + 16;
  for (int c = 0; c < 4; ++c) {
    for (int l = 0; l < 32; ++l) {
      qs[32 * c + l] = static_cast<uint8_t>(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
  }
}

// One Q6_K super-block: value = d*sc[j]*(q-32), q in 0..63, 16 sub-blocks of 16.
void QuantizeQ6K(const float* x, uint8_t* out) {
  float s[16];
  float smax = 0.f;
  for (int j = 0; j < 16; ++j) {
    float a = 0.f;
    for (int i = 0; i < 16; ++i) a = std::max(a, std::fabs(x[16 * j + i]));
    s[j] = a / 31.f;
    smax = std::max(smax, s[j]);
  }
  const uint16_t dh = ToHalf(smax / 127.f);
  const float d = FromHalf(dh);
  int sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = d > 0 ? RoundClamp(s[j] / d, -128, 127) : 0;
  int q[kQK];
  for (int j = 0; j < 16; ++j) {
    const float step = d * sc[j];
    for (int i = 0; i < 16; ++i) {
      q[16 * j + i] = (step > 0 ? RoundClamp(x[16 * j + i] / step, -32, 31) : 0) + 32;
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  int8_t* scales = reinterpret_cast<int8_t*>(out + 192);
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      const int q1 = q[128 * h + l], q2 = q[128 * h + 32 + l];
      const int q3 = q[128 * h + 64 + l], q4 = q[128 * h + 96 + l];
      ql[64 * h + l] = static_cast<uint8_t>((q1 & 15) | ((q3 & 15) << 4));
      ql[64 * h + 32 + l] = static_cast<uint8_t>((q2 & 15) | ((q4 & 15) << 4));
      qh[32 * h + l] = static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) |
                                            ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  for (int j = 0; j < 16; ++j) scales[j] = static_cast<int8_t>(sc[j]);
  std::memcpy(out + 208, &dh, 2);
}

}  // namespace

extern "C" {

// Layout must match nuthatch_b200/synth.py (ctypes Structure).
struct NhSynthSpec {
  uint32_t n_layers;
  uint32_t n_embd;
  uint32_t n_head;
  uint32_t n_head_kv;
  uint32_t n_ff;
  uint32_t n_expert;
  uint32_t n_expert_used;
  uint32_t n_vocab;
  uint32_t n_ctx_train;
  float rope_freq_base;
  float rms_eps;
  float weight_std;
  uint64_t seed;
  int32_t quant;        // 0: every tensor F32; 1: Q4_K_M-like mix
  float skew_embd;      // constant written into column 0 of every token_embd row (0: off)
  float skew_router;    // router column-0 gain: row e gets skew_router * beta_e
  float skew_zipf_s;    // log-Zipf exponent for beta_e = -s*ln(rank_e); 0: off
  int32_t n_threads;    // 0: hardware concurrency
};

}  // extern "C"

namespace {

struct TensorPlan {
  std::string name;
  std::vector<uint64_t> ne;
  uint32_t type;
  uint64_t offset = 0;
  uint64_t nbytes = 0;
  int kind = 0;  // 0 weight, 1 norm (ones), 2 router, 3 token_embd
};

uint64_t RowBytes(uint32_t type, uint64_t ne0) {
  if (type == kTypeQ4K) return ne0 / kQK * kQ4KBytes;
  if (type == kTypeQ6K) return ne0 / kQK * kQ6KBytes;
  return ne0 * 4;
}

struct Writer {
  FILE* f;
  bool ok = true;
  void Raw(const void* p, size_t n) {
    if (ok && std::fwrite(p, 1, n, f) != n) ok = false;
  }
  void U32(uint32_t v) { Raw(&v, 4); }
  void U64(uint64_t v) { Raw(&v, 8); }
  void F32(float v) { Raw(&v, 4); }
  void Str(const std::string& s) {
    U64(s.size());
    Raw(s.data(), s.size());
  }
  void KvU32(const std::string& k, uint32_t v) {
    Str(k);
    U32(4);  // GGUF_TYPE_UINT32
    U32(v);
  }
  void KvF32(const std::string& k, float v) {
    Str(k);
    U32(6);  // GGUF_TYPE_FLOAT32
    F32(v);
  }
  void KvStr(const std::string& k, const std::string& v) {
    Str(k);
    U32(8);  // GGUF_TYPE_STRING
    Str(v);
  }
};

void ParallelFor(int64_t n, int threads, const std::function<void(int64_t, int64_t)>& fn) {
  if (threads <= 1 || n < 64) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> ts;
  std::atomic<int64_t> next{0};
  const int64_t chunk = std::max<int64_t>(1, n / (threads * 8));
  for (int t = 0; t < threads; ++t) {
    ts.emplace_back([&]() {
      for (;;) {
        const int64_t b = next.fetch_add(chunk);
        if (b >= n) break;
        fn(b, std::min(n, b + chunk));
      }
    });
  }
  for (auto& t : ts) t.join();
}

}  // namespace

extern "C" int nh_synth_write_olmoe(const char* path, const NhSynthSpec* sp) {
  if (path == nullptr || sp == nullptr) return -1;
  const NhSynthSpec& s = *sp;
  if (s.n_layers == 0 || s.n_embd == 0 || s.n_head == 0 || s.n_ff == 0 ||
      s.n_expert == 0 || s.n_vocab == 0 || s.n_embd % s.n_head != 0) {
    return -2;
  }
  const uint32_t head_kv = s.n_head_kv ? s.n_head_kv : s.n_head;
  const uint64_t d = s.n_embd, F = s.n_ff, E = s.n_expert, V = s.n_vocab;
  const uint64_t dkv = static_cast<uint64_t>(head_kv) * (d / s.n_head);
  int threads = s.n_threads > 0 ? s.n_threads
                                : static_cast<int>(std::thread::hardware_concurrency());
  if (threads <= 0) threads = 4;

  auto qtype = [&](uint32_t want, uint64_t ne0) -> uint32_t {
    if (s.quant == 0 || ne0 % kQK != 0) return kTypeF32;
    return want;
  };

  std::vector<TensorPlan> plan;
  auto add = [&](const std::string& name, std::vector<uint64_t> ne, uint32_t type, int kind) {
    TensorPlan t;
    t.name = name;
    t.ne = std::move(ne);
    t.type = type;
    t.kind = kind;
    uint64_t rows = 1;
    for (size_t i = 1; i < t.ne.size(); ++i) rows *= t.ne[i];
    t.nbytes = RowBytes(type, t.ne[0]) * rows;
    plan.push_back(t);
  };
  add("token_embd.weight", {d, V}, qtype(kTypeQ4K, d), 3);
  for (uint32_t l = 0; l < s.n_layers; ++l) {
    const std::string b = "blk." + std::to_string(l) + ".";
    const bool odd = (l % 2) == 1;
    add(b + "attn_norm.weight", {d}, kTypeF32, 1);
    add(b + "attn_q.weight", {d, d}, qtype(kTypeQ4K, d), 0);
    add(b + "attn_k.weight", {d, dkv}, qtype(kTypeQ4K, d), 0);
    add(b + "attn_v.weight", {d, dkv}, qtype(odd ? kTypeQ6K : kTypeQ4K, d), 0);
    add(b + "attn_output.weight", {d, d}, qtype(kTypeQ4K, d), 0);
    add(b + "attn_q_norm.weight", {d}, kTypeF32, 1);
    add(b + "attn_k_norm.weight", {dkv}, kTypeF32, 1);
    add(b + "ffn_norm.weight", {d}, kTypeF32, 1);
    add(b + "ffn_gate_inp.weight", {d, E}, kTypeF32, 2);
    add(b + "ffn_gate_exps.weight", {d, F, E}, qtype(kTypeQ4K, d), 0);
    add(b + "ffn_up_exps.weight", {d, F, E}, qtype(kTypeQ4K, d), 0);
    add(b + "ffn_down_exps.weight", {F, d, E}, qtype(odd ? kTypeQ6K : kTypeQ4K, F), 0);
  }
  add("output_norm.weight", {d}, kTypeF32, 1);
  add("output.weight", {d, V}, qtype(kTypeQ6K, d), 0);

  uint64_t off = 0;
  for (auto& t : plan) {
    t.offset = off;
    off += (t.nbytes + kAlign - 1) / kAlign * kAlign;
  }

  // Router bias ranks for the log-Zipf skew: a seeded permutation of 0..E-1.
  std::vector<float> beta(E, 0.f);
  if (s.skew_zipf_s > 0.f) {
    std::vector<uint32_t> perm(E);
    for (uint32_t e = 0; e < E; ++e) perm[e] = e;
    uint64_t st = Mix64(s.seed ^ 0x5a5a5a5aull);
    for (uint32_t i = E - 1; i > 0; --i) {
      st = Mix64(st);
      const uint32_t j = static_cast<uint32_t>(st % (i + 1));
      std::swap(perm[i], perm[j]);
    }
    for (uint32_t r = 0; r < E; ++r) {
      beta[perm[r]] = -s.skew_zipf_s * std::log(static_cast<float>(r + 1));
    }
  }

  FILE* f = std::fopen(path, "wb");
  if (f == nullptr) return -3;
  Writer w{f};
  w.Raw("GGUF", 4);
  w.U32(3);
  w.U64(plan.size());
  w.U64(12);
  w.KvStr("general.architecture", "olmoe");
  w.KvU32("olmoe.block_count", s.n_layers);
  w.KvU32("olmoe.embedding_length", s.n_embd);
  w.KvU32("olmoe.attention.head_count", s.n_head);
  w.KvU32("olmoe.attention.head_count_kv", head_kv);
  w.KvU32("olmoe.feed_forward_length", s.n_ff);
  w.KvU32("olmoe.expert_count", s.n_expert);
  w.KvU32("olmoe.expert_used_count", s.n_expert_used);
  w.KvU32("olmoe.context_length", s.n_ctx_train);
  w.KvF32("olmoe.rope.freq_base", s.rope_freq_base);
  w.KvF32("olmoe.attention.layer_norm_rms_epsilon", s.rms_eps);
  w.KvU32("general.alignment", static_cast<uint32_t>(kAlign));
  for (const auto& t : plan) {
    w.Str(t.name);
    w.U32(static_cast<uint32_t>(t.ne.size()));
    for (uint64_t n : t.ne) w.U64(n);
    w.U32(t.type);
    w.U64(t.offset);
  }
  long pos = std::ftell(f);
  const long pad = (kAlign - pos % kAlign) % kAlign;
  static const char zeros[64] = {0};
  w.Raw(zeros, static_cast<size_t>(pad));

  std::vector<uint8_t> buf;
  for (const auto& t : plan) {
    buf.assign((t.nbytes + kAlign - 1) / kAlign * kAlign, 0);
    const uint64_t ne0 = t.ne[0];
    uint64_t rows = 1;
    for (size_t i = 1; i < t.ne.size(); ++i) rows *= t.ne[i];
    const uint64_t rb = RowBytes(t.type, ne0);
    const uint64_t tseed = Mix64(s.seed ^ HashName(t.name));
    const float stdv = s.weight_std;
    const int kind = t.kind;
    const uint32_t type = t.type;
    uint8_t* base = buf.data();
    ParallelFor(static_cast<int64_t>(rows), threads, [&](int64_t r0, int64_t r1) {
      std::vector<float> row(ne0);
      for (int64_t r = r0; r < r1; ++r) {
        for (uint64_t i = 0; i < ne0; ++i) {
          if (kind == 1) {
            row[i] = 1.0f;
          } else {
            row[i] = stdv * NormalApprox(tseed + static_cast<uint64_t>(r) * ne0 + i);
          }
        }
        if (kind == 3 && s.skew_embd != 0.f) row[0] = s.skew_embd;
        if (kind == 2 && s.skew_zipf_s > 0.f) {
          row[0] = s.skew_router * beta[static_cast<uint64_t>(r) % E];
        }
        uint8_t* dst = base + static_cast<uint64_t>(r) * rb;
        if (type == kTypeQ4K) {
          for (uint64_t b = 0; b < ne0 / kQK; ++b) QuantizeQ4K(&row[b * kQK], dst + b * kQ4KBytes);
        } else if (type == kTypeQ6K) {
          for (uint64_t b = 0; b < ne0 / kQK; ++b) QuantizeQ6K(&row[b * kQK], dst + b * kQ6KBytes);
        } else {
          std::memcpy(dst, row.data(), ne0 * 4);
        }
      }
    });
    w.Raw(buf.data(), buf.size());
    if (!w.ok) break;
  }
  const bool ok = w.ok;
  if (std::fclose(f) != 0 || !ok) return -4;
  return 0;
}

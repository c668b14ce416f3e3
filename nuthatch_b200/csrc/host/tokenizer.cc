// GPT-2 byte-level BPE tokenizer (reference: src/tokenizer/tokenizer.cc).
// Own design: a hand-written matcher of the OLMo pre-split pattern over
// generated Unicode category ranges (no regex engine), and BPE merges driven
// by a min-heap over a linked list of symbols (the reference rescans every
// adjacent pair per merge; the order of merges is the same).
#include "nuthatch/tokenizer.h"

#include <algorithm>
#include <queue>

#include "nuthatch/gguf_file.h"

namespace nuthatch {
namespace {

struct CodeRange {
  uint32_t lo, hi;
};

#include "unicode_tables.inc"

template <size_t N>
bool InRanges(const CodeRange (&r)[N], uint32_t cp) {
  const CodeRange* end = r + N;
  const CodeRange* it = std::upper_bound(r, end, cp, [](uint32_t v, const CodeRange& x) { return v < x.lo; });
  return it != r && cp <= (it - 1)->hi;
}

// Classes of the pre-split pattern: \s, \p{L}, \p{N}, and everything else.
enum class Cls { kSpace, kLetter, kNumber, kOther };

Cls Classify(uint32_t cp) {
  if (cp < 0x80) {
    if ((cp >= 'a' && cp <= 'z') || (cp >= 'A' && cp <= 'Z')) return Cls::kLetter;
    if (cp >= '0' && cp <= '9') return Cls::kNumber;
    if (cp == ' ' || (cp >= 0x09 && cp <= 0x0D)) return Cls::kSpace;
    return Cls::kOther;
  }
  if (InRanges(kSeparatorRanges, cp)) return Cls::kSpace;
  if (InRanges(kLetterRanges, cp)) return Cls::kLetter;
  if (InRanges(kNumberRanges, cp)) return Cls::kNumber;
  return Cls::kOther;
}

// One code point of valid UTF-8 at p[0..n): its length (1-4), or 0 when the
// bytes there are not a well-formed sequence (overlong forms, surrogates and
// values above U+10FFFF are not).
int DecodeUtf8(const unsigned char* p, size_t n, uint32_t* cp) {
  const unsigned c = p[0];
  int len;
  uint32_t v, min;
  if (c < 0x80) {
    *cp = c;
    return 1;
  } else if ((c & 0xE0) == 0xC0) {
    len = 2, v = c & 0x1F, min = 0x80;
  } else if ((c & 0xF0) == 0xE0) {
    len = 3, v = c & 0x0F, min = 0x800;
  } else if ((c & 0xF8) == 0xF0) {
    len = 4, v = c & 0x07, min = 0x10000;
  } else {
    return 0;
  }
  if (n < static_cast<size_t>(len)) return 0;
  for (int i = 1; i < len; ++i) {
    if ((p[i] & 0xC0) != 0x80) return 0;
    v = (v << 6) | (p[i] & 0x3F);
  }
  if (v < min || v > 0x10FFFF || (v >= 0xD800 && v <= 0xDFFF)) return 0;
  *cp = v;
  return len;
}

// The text as code points with their byte offsets (offsets has one more
// entry: the end).  false when the text is not valid UTF-8.
bool CodePoints(const std::string& text, std::vector<uint32_t>* cps, std::vector<size_t>* offsets) {
  const auto* p = reinterpret_cast<const unsigned char*>(text.data());
  cps->clear();
  offsets->clear();
  for (size_t i = 0; i < text.size();) {
    uint32_t cp = 0;
    const int len = DecodeUtf8(p + i, text.size() - i, &cp);
    if (len == 0) return false;
    cps->push_back(cp);
    offsets->push_back(i);
    i += static_cast<size_t>(len);
  }
  offsets->push_back(text.size());
  return true;
}

// The byte-level character of each byte (GPT-2's table): the printable bytes
// '!'..'~', 0xA1..0xAC and 0xAE..0xFF stand for themselves; the other 68
// bytes take the code points 256, 257, ... in byte order.
uint32_t ByteLevelCodePoint(int b, int* next_extra) {
  const bool printable = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
  return printable ? static_cast<uint32_t>(b) : static_cast<uint32_t>(256 + (*next_extra)++);
}

std::string EncodeUtf8(uint32_t cp) {
  std::string s;
  if (cp < 0x80) {
    s += static_cast<char>(cp);
  } else if (cp < 0x800) {
    s += static_cast<char>(0xC0 | (cp >> 6));
    s += static_cast<char>(0x80 | (cp & 0x3F));
  } else {
    s += static_cast<char>(0xE0 | (cp >> 12));
    s += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
    s += static_cast<char>(0x80 | (cp & 0x3F));
  }
  return s;
}

}  // namespace

namespace {

// The end (code-point index) of the pre-split pattern's match starting at
// code point s, or s when no alternative matches there.  The alternatives
// are tried in the pattern's order and the first that matches is taken:
//   1. 's 't 're 've 'm 'll 'd          (ASCII apostrophe, lower case)
//   2-4. an optional U+0020, then one or more letters / numbers / others
//        (each run as long as possible; without a fitting character after
//        the space the optional space cannot start the run either)
//   5. \s+(?!\S): a whitespace run that ends the text, or the run minus
//      its last character when a non-space follows and the run is longer
//      than one.
size_t MatchAt(const std::vector<uint32_t>& cp, const std::vector<Cls>& cls, size_t s) {
  const size_t n = cp.size();
  if (cp[s] == '\'') {
    static const char* const kSuffix[] = {"s", "t", "re", "ve", "m", "ll", "d"};
    for (const char* suf : kSuffix) {
      size_t i = s + 1, k = 0;
      while (suf[k] != '\0' && i < n && cp[i] == static_cast<unsigned char>(suf[k])) ++i, ++k;
      if (suf[k] == '\0') return i;
    }
  }
  const size_t run_from = cp[s] == ' ' && s + 1 < n ? s + 1 : s;
  for (Cls c : {Cls::kLetter, Cls::kNumber, Cls::kOther}) {
    size_t e = run_from;
    while (e < n && cls[e] == c) ++e;
    if (e > run_from) return e;
  }
  if (cls[s] == Cls::kSpace) {
    size_t e = s;
    while (e < n && cls[e] == Cls::kSpace) ++e;
    if (e == n) return e;
    if (e - s >= 2) return e - 1;
  }
  return s;
}

}  // namespace

std::vector<std::pair<size_t, size_t>> Tokenizer::Split(const std::string& text) {
  std::vector<std::pair<size_t, size_t>> chunks;
  std::vector<uint32_t> cp;
  std::vector<size_t> at;
  if (!CodePoints(text, &cp, &at)) return chunks;
  std::vector<Cls> cls(cp.size());
  for (size_t i = 0; i < cp.size(); ++i) cls[i] = Classify(cp[i]);
  // Each search starts where the previous match ended and takes the first
  // position from there at which the pattern matches; what it passes over
  // belongs to no chunk.
  for (size_t s = 0; s < cp.size();) {
    const size_t e = MatchAt(cp, cls, s);
    if (e == s) {
      ++s;
      continue;
    }
    chunks.emplace_back(at[s], at[e]);
    s = e;
  }
  return chunks;
}

Tokenizer::Tokenizer(std::vector<std::string> vocab, std::vector<std::string> merges) : vocab_(std::move(vocab)) {
  std::unordered_map<std::string, int> sym_of;
  auto intern = [&](const std::string& text) {
    return sym_of.emplace(text, static_cast<int>(sym_of.size())).first->second;
  };
  int extra = 0;
  for (int b = 0; b < 256; ++b) {
    const uint32_t cp = ByteLevelCodePoint(b, &extra);
    byte_sym_[b] = intern(EncodeUtf8(cp));
    char_byte_[cp] = static_cast<uint8_t>(b);
  }
  for (const std::string& v : vocab_) intern(v);
  for (size_t r = 0; r < merges.size(); ++r) {
    const std::string& m = merges[r];
    const size_t sp = m.find(' ');
    if (sp == std::string::npos || sp == 0 || sp + 1 == m.size() || m.find(' ', sp + 1) != std::string::npos) continue;
    const std::string a = m.substr(0, sp), b = m.substr(sp + 1);
    const uint64_t key = static_cast<uint64_t>(intern(a)) << 32 | static_cast<uint32_t>(intern(b));
    const int ab = intern(a + b);
    merge_.emplace(key, std::make_pair(static_cast<int>(r), ab));  // the first rank of a pair stays
  }
  // The first occurrence of a vocabulary string keeps its id.
  sym_id_.assign(sym_of.size(), -1);
  for (size_t i = 0; i < vocab_.size(); ++i) {
    int32_t& id = sym_id_[sym_of.at(vocab_[i])];
    if (id < 0) id = static_cast<int32_t>(i);
  }
}

Tokenizer::~Tokenizer() = default;

std::unique_ptr<Tokenizer> Tokenizer::FromLists(std::vector<std::string> vocab, std::vector<std::string> merges) {
  return std::unique_ptr<Tokenizer>(new Tokenizer(std::move(vocab), std::move(merges)));
}

std::unique_ptr<Tokenizer> Tokenizer::Load(const std::string& path) {
  static const std::vector<std::string> kKeys = {"tokenizer.ggml.tokens", "tokenizer.ggml.merges"};
  std::unordered_map<std::string, std::vector<std::string>> arrays;
  if (!ReadGgufStringArrays(path, kKeys, &arrays)) return nullptr;
  auto tokens = arrays.find(kKeys[0]);
  if (tokens == arrays.end()) return nullptr;
  auto merges = arrays.find(kKeys[1]);
  return FromLists(std::move(tokens->second), merges != arrays.end() ? std::move(merges->second)
                                                                     : std::vector<std::string>());
}

const std::string& Tokenizer::token(int32_t id) const {
  static const std::string kNone;
  return id >= 0 && static_cast<size_t>(id) < vocab_.size() ? vocab_[id] : kNone;
}

// BPE over one chunk: its bytes become byte-level symbols in a linked list;
// a min-heap holds every adjacent pair that has a merge, keyed by (rank,
// position of the left symbol), so the pair merged next is the lowest rank,
// leftmost among equal ranks, as a full rescan would pick.  Entries made
// stale by an earlier merge are recognised by the symbols' versions.  Chunks
// seen before take their ids from the cache.
void Tokenizer::EncodeChunk(const char* p, size_t n, std::vector<int32_t>* out) const {
  if (n == 0) return;
  const std::string chunk(p, n);
  {
    std::lock_guard<std::mutex> hold(cache_mu_);
    auto hit = cache_.find(chunk);
    if (hit != cache_.end()) {
      out->insert(out->end(), hit->second.begin(), hit->second.end());
      return;
    }
  }
  struct Sym {
    int sym, prev, next;
    unsigned version;
  };
  std::vector<Sym> sym(n);
  for (size_t i = 0; i < n; ++i)
    sym[i] = {byte_sym_[static_cast<unsigned char>(p[i])], static_cast<int>(i) - 1,
              i + 1 < n ? static_cast<int>(i) + 1 : -1, 0};
  struct Cand {
    int rank, left, right, merged;
    unsigned vl, vr;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : left > o.left; }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto offer = [&](int l) {
    const int r = l >= 0 ? sym[l].next : -1;
    if (r < 0) return;
    auto it = merge_.find(static_cast<uint64_t>(sym[l].sym) << 32 | static_cast<uint32_t>(sym[r].sym));
    if (it != merge_.end()) heap.push({it->second.first, l, r, it->second.second, sym[l].version, sym[r].version});
  };
  for (int i = 0; i + 1 < static_cast<int>(n); ++i) offer(i);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    Sym& L = sym[c.left];
    Sym& R = sym[c.right];
    if (L.next != c.right || L.version != c.vl || R.version != c.vr) continue;
    L.sym = c.merged;
    ++L.version;
    ++R.version;  // R leaves the list
    L.next = R.next;
    if (R.next >= 0) sym[R.next].prev = c.left;
    offer(L.prev);
    offer(c.left);
  }
  std::vector<int32_t> ids;
  for (int i = 0; i >= 0; i = sym[i].next)
    if (sym_id_[sym[i].sym] >= 0) ids.push_back(sym_id_[sym[i].sym]);
  out->insert(out->end(), ids.begin(), ids.end());
  std::lock_guard<std::mutex> hold(cache_mu_);
  if (cache_.size() >= (1u << 16)) cache_.clear();
  cache_.emplace(chunk, std::move(ids));
}

std::vector<int32_t> Tokenizer::Encode(const std::string& text) const {
  std::vector<int32_t> ids;
  for (const auto& ch : Split(text)) EncodeChunk(text.data() + ch.first, ch.second - ch.first, &ids);
  return ids;
}

// Decode reads each vocabulary string with the reference's rules
// (tokenizer.cc:33-48, 188-200): a lead byte 110xxxxx or 1110xxxx with enough
// bytes after it takes one or two following bytes whatever they are; any
// other byte stands for the code point of its own value.  A code point that
// is no byte-level character adds nothing.
std::string Tokenizer::Decode(const std::vector<int32_t>& ids) const {
  std::string out;
  for (int32_t id : ids) {
    if (id < 0 || static_cast<size_t>(id) >= vocab_.size()) continue;
    const std::string& t = vocab_[id];
    const size_t n = t.size();
    for (size_t i = 0; i < n;) {
      const unsigned c = static_cast<unsigned char>(t[i]);
      uint32_t cp = c;
      size_t len = 1;
      if ((c >> 5) == 0x6 && i + 1 < n) {
        cp = ((c & 0x1Fu) << 6) | (static_cast<unsigned char>(t[i + 1]) & 0x3Fu);
        len = 2;
      } else if ((c >> 4) == 0xE && i + 2 < n) {
        cp = ((c & 0x0Fu) << 12) | ((static_cast<unsigned char>(t[i + 1]) & 0x3Fu) << 6) |
             (static_cast<unsigned char>(t[i + 2]) & 0x3Fu);
        len = 3;
      }
      i += len;
      auto it = char_byte_.find(cp);
      if (it != char_byte_.end()) out += static_cast<char>(it->second);
    }
  }
  return out;
}

}  // namespace nuthatch
